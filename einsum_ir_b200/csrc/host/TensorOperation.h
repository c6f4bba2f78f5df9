// TensorOperation: the explicit-descriptor front door of the reference's etops
// package (python/src/TensorOperation.h:29-421, TensorOperation.cpp:1-771):
// one binary contraction (prim_main gemm / brgemm) or one unary operation
// (copy / zero) given by dimension types, execution types, sizes and a
// [LEVEL][TENSOR][DIMENSION] stride tensor, set up once and executed on
// device pointers.
//
// Same enums, values, error codes and validation order as the reference. The
// execution maps onto the backend's C-ABI plans: a binary operation becomes
// one eir_contract plan (the planner picks tcgen05 / DMMA / CUDA-core
// kernels), a unary one an eir_unary plan. Execution types and level-1
// packing strides are scheduling hints of the CPU backend: they are accepted
// with the reference's shape rules and do not change the result, which the
// GPU kernels compute from the level-0 strides alone.
#ifndef EINSUM_IR_B200_TENSOR_OPERATION_H
#define EINSUM_IR_B200_TENSOR_OPERATION_H

#include <cstdint>
#include <tuple>
#include <vector>

struct eir_plan;

namespace einsum_ir {
namespace py {

//! backend optimisation parameters (python/src/TensorOperation.h:17-27)
struct OptimizationConfig {
  int64_t target_m = 0;
  int64_t target_n = 0;
  int64_t target_k = 0;
  int64_t num_threads = 0;
  bool br_gemm_support = false;
  bool packed_gemm_support = false;
  bool packing_support = false;
  bool sfc_support = false;
  int64_t l2_cache_size = 0;
};

class TensorOperation {
 public:
  enum class op_type_t : uint32_t { binary = 0, unary = 1, undefined = 99 };
  enum class exec_t : uint32_t { seq = 0, prim = 1, shared = 2, sfc = 3, undefined = 99 };
  enum class prim_t : uint32_t { none = 0, zero = 1, copy = 2, relu = 3, gemm = 4, brgemm = 5, undefined = 99 };
  enum class dim_t : uint32_t { c = 0, m = 1, n = 2, k = 3, undefined = 99 };
  enum class dtype_t : uint32_t { fp32 = 0, fp64 = 1 };
  enum class error_t : int32_t {
    success = 0,
    compilation_failed = 1,
    invalid_stride_shape = 2,
    invalid_optimization_config = 3
  };
  using strides_t = std::vector<std::vector<std::vector<int64_t>>>;

  TensorOperation() = default;
  ~TensorOperation();
  TensorOperation(TensorOperation const &) = delete;
  TensorOperation &operator=(TensorOperation const &) = delete;

  //! set-up of a binary contraction or a unary operation (the type follows
  //! from prim_main); strides in elements
  error_t setup(dtype_t dtype, prim_t prim_first, prim_t prim_main, prim_t prim_last,
                std::vector<dim_t> const &dim_types, std::vector<exec_t> const &exec_types,
                std::vector<int64_t> const &dim_sizes, strides_t const &strides);

  //! runs the operation on device pointers (in1 unused for unary operations),
  //! asynchronously on the operation's stream
  void execute(void const *tensor_in0, void const *tensor_in1, void *tensor_out);

  //! returns a configuration describing how the B200 backend executes the
  //! operation: size-1 dims dropped, dims that are contiguous in every tensor
  //! fused, execution types set to the kernels' mapping (prim: the tile
  //! dims of the kernel; shared: dims spread over CTAs; seq: the K loop),
  //! a single stride level (the kernels read operands in place)
  static std::tuple<error_t, dtype_t, prim_t, prim_t, prim_t, std::vector<dim_t>, std::vector<exec_t>,
                    std::vector<int64_t>, strides_t>
  optimize(dtype_t dtype, prim_t prim_first, prim_t prim_main, prim_t prim_last,
           std::vector<dim_t> const &dim_types, std::vector<exec_t> const &exec_types,
           std::vector<int64_t> const &dim_sizes, strides_t const &strides,
           OptimizationConfig const &optimization_config);

  //! the reference's defaults (python/src/TensorOperation.cpp:470-481)
  static OptimizationConfig get_default_optimization_config();

  //! extensions of this backend: stream for execute, the status of the last
  //! execute (an eir status), the plan (for eir_plan_* queries)
  void set_stream(void *i_stream) { m_stream = i_stream; }
  int last_status() const { return m_status; }
  eir_plan const *plan() const { return m_plan; }
  op_type_t op_type() const { return m_op_type; }

  static op_type_t determine_op_type(prim_t prim_main);

 private:
  void release();
  op_type_t m_op_type = op_type_t::undefined;
  eir_plan *m_plan = nullptr;
  void *m_stream = nullptr;
  int m_status = 0;
};

}  // namespace py
}  // namespace einsum_ir

#endif
