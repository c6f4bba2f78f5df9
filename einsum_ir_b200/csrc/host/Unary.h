// Unary permute-copy between dim orders of one tensor.
// Interface of the reference's backend::Unary (src/backend/Unary.h:16-156):
// init(num_dims, sizes, ids_in, ids_out, dtypes, ktype, threads), compile, eval.
// UnaryCuda lowers it to the C-ABI permute plan (eir_permute_plan_create) and
// runs it on the backend's stream.
#ifndef EINSUM_IR_B200_UNARY_H
#define EINSUM_IR_B200_UNARY_H

#include <cstdint>
#include <map>
#include <vector>
#include "constants.h"
#include "eir_cuda.h"

namespace einsum_ir {
namespace backend {

class Unary {
 public:
  int64_t m_num_dims = 0;
  std::map<int64_t, int64_t> const *m_dim_sizes = nullptr;
  int64_t const *m_dim_ids_in = nullptr;
  int64_t const *m_dim_ids_out = nullptr;
  data_t m_dtype_in = UNDEFINED_DTYPE, m_dtype_comp = UNDEFINED_DTYPE, m_dtype_out = UNDEFINED_DTYPE;
  kernel_t m_ktype_main = UNDEFINED_KTYPE;
  int64_t m_num_threads = 1;
  bool m_compiled = false;
  //! strides of the input tensor w.r.t. the output's dim order, and of the output
  std::vector<int64_t> m_strides_in, m_strides_out;

  //! row-major strides of a tensor (reference Unary.cpp:3-14)
  static void strides(int64_t i_num_dims, std::map<int64_t, int64_t> const *i_dim_sizes,
                      int64_t const *i_dim_ids, int64_t *o_strides);
  //! reorders input strides to the output's dim order (reference Unary.cpp:16-31)
  static void order_strides_output_based(int64_t i_num_dims, int64_t const *i_dim_ids_in,
                                         int64_t const *i_dim_ids_out, int64_t *io_strides);

  virtual ~Unary() {}
  void init(int64_t i_num_dims, std::map<int64_t, int64_t> const *i_dim_sizes,
            int64_t const *i_dim_ids_in, int64_t const *i_dim_ids_out, data_t i_dtype_in,
            data_t i_dtype_comp, data_t i_dtype_out, kernel_t i_ktype_main, int64_t i_num_threads);
  virtual err_t compile() = 0;
  virtual void eval(void const *i_tensor_in, void *io_tensor_out) = 0;
};

class UnaryCuda : public Unary {
 public:
  ~UnaryCuda() override;
  err_t compile() override;
  void eval(void const *i_tensor_in, void *io_tensor_out) override;
  void set_stream(void *i_stream) { m_stream = i_stream; }
  int m_last_status = EIR_SUCCESS;
  eir_plan *m_plan = nullptr;

 private:
  void *m_stream = nullptr;
};

}  // namespace backend
}  // namespace einsum_ir

#endif
