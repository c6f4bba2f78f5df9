// B200 backend of the binary contraction interface: compile() lowers the dim
// analysis of BinaryContraction to the C-ABI descriptor (eir_contract_desc)
// and creates a plan; contract() enqueues it on the backend's stream.
// Replaces the reference's BinaryContractionTpp (src/backend/BinaryContractionTpp.cpp:4-147).
#ifndef EINSUM_IR_B200_BINARY_CONTRACTION_CUDA_H
#define EINSUM_IR_B200_BINARY_CONTRACTION_CUDA_H

#include "BinaryContraction.h"
#include "eir_cuda.h"

namespace einsum_ir {
namespace backend {

class BinaryContractionCuda : public BinaryContraction {
 public:
  ~BinaryContractionCuda() override;

  //! compute type used by compile (EIR_COMPUTE_*; default: exact for the data type)
  void set_compute_type(int32_t i_comp) { m_comp = i_comp; }
  //! stream the contraction is enqueued on (cudaStream_t; nullptr = legacy default)
  void set_stream(void *i_stream) { m_stream = i_stream; }
  //! planner flags (EIR_FLAG_*)
  void set_flags(int32_t i_flags) { m_flags = i_flags; }

  err_t compile() override;
  void contract(void const *i_tensor_left, void const *i_tensor_right, void *io_tensor_out) override;
  void contract(void const *i_tensor_left, void const *i_tensor_right, void const *i_tensor_out_aux,
                void *io_tensor_out) override;

  //! status of the last contract call (EIR_*; contract itself returns nothing, as in the reference)
  int m_last_status = EIR_SUCCESS;
  eir_plan *m_plan = nullptr;

 private:
  int32_t m_comp = EIR_COMPUTE_DEFAULT;
  int32_t m_flags = 0;
  void *m_stream = nullptr;
};

}  // namespace backend
}  // namespace einsum_ir

#endif
