/*
 * eir_tensor_operation.h -- C-ABI of the explicit-descriptor tensor operation
 * (the reference's etops front door, python/src/TensorOperation.h:29-421 and
 * its pybind11 module python/src/bindings.cpp:14-334).
 *
 * Enum values are the reference's: dtype 0 = fp32, 1 = fp64; prim 0 none,
 * 1 zero, 2 copy, 3 relu, 4 gemm, 5 brgemm; exec 0 seq, 1 prim, 2 shared,
 * 3 sfc; dim 0 c, 1 m, 2 n, 3 k. eir_top_setup and eir_top_optimize return
 * the reference's error_t (0 success, 1 compilation_failed,
 * 2 invalid_stride_shape, 3 invalid_optimization_config); the other calls
 * return eir status codes (eir_cuda.h).
 *
 * Strides are passed flattened in [LEVEL][TENSOR][DIMENSION] order: level l
 * holds tensors_per_level[l] vectors, vector v (counted over all levels) has
 * dims_per_vector[v] entries. Level 0 must hold 3 vectors (binary: in0, in1,
 * out) or 2 (unary: in, out) of num_dims strides each; a level 1 of 3 vectors
 * is the reference's packing level (accepted; it does not change the result).
 *
 * Reference interfaces replaced:
 *   eir_top_setup      <- TensorOperation::setup (TensorOperation.h:104-113)
 *   eir_top_execute    <- TensorOperation::execute (TensorOperation.h:122-124)
 *   eir_top_optimize   <- TensorOperation::optimize (TensorOperation.h:144-164)
 *   eir_top_default_optimization_config
 *                      <- TensorOperation::get_default_optimization_config (:172)
 */
#ifndef EIR_TENSOR_OPERATION_H
#define EIR_TENSOR_OPERATION_H

#include <stdint.h>
#include "eir_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct eir_tensor_operation eir_tensor_operation;

typedef struct {
  int64_t target_m;
  int64_t target_n;
  int64_t target_k;
  int64_t num_threads;
  int32_t br_gemm_support;
  int32_t packed_gemm_support;
  int32_t packing_support;
  int32_t sfc_support;
  int64_t l2_cache_size;
} eir_top_optimization_config;

int eir_top_create(eir_tensor_operation **op);
int eir_top_destroy(eir_tensor_operation *op);
int eir_top_setup(eir_tensor_operation *op, int32_t dtype, int32_t prim_first, int32_t prim_main,
                  int32_t prim_last, int32_t num_dims, int32_t const *dim_types,
                  int32_t const *exec_types, int64_t const *dim_sizes, int32_t num_levels,
                  int32_t const *tensors_per_level, int32_t const *dims_per_vector,
                  int64_t const *strides);
/* device pointers; in1 is ignored (may be NULL) for unary operations;
 * asynchronous on `stream` (a cudaStream_t, NULL = legacy default stream) */
int eir_top_execute(eir_tensor_operation *op, void const *in0, void const *in1, void *out,
                    void *stream);
/* the plan behind a set-up operation (for eir_plan_kernel_family and the
 * like), NULL before a successful set-up */
eir_plan const *eir_top_plan(eir_tensor_operation const *op);
int eir_top_default_optimization_config(eir_top_optimization_config *cfg);
/* outputs: the optimised descriptor, one stride level. Capacities: num_dims
 * entries for the per-dim arrays and 3 * num_dims strides (the optimisation
 * never adds dims). out_tensors: number of stride vectors of the level. */
int eir_top_optimize(int32_t dtype, int32_t prim_first, int32_t prim_main, int32_t prim_last,
                     int32_t num_dims, int32_t const *dim_types, int32_t const *exec_types,
                     int64_t const *dim_sizes, int32_t num_levels, int32_t const *tensors_per_level,
                     int32_t const *dims_per_vector, int64_t const *strides,
                     eir_top_optimization_config const *cfg, int32_t *out_num_dims,
                     int32_t *out_dim_types, int32_t *out_exec_types, int64_t *out_dim_sizes,
                     int32_t *out_tensors, int64_t *out_strides);

#ifdef __cplusplus
}
#endif

#endif
