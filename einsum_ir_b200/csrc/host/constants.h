// Enumerations of the einsum_ir host API (values as in the reference's
// src/constants.h:8-87, so code written against the reference compiles and
// behaves the same). Extensions for this backend: data_t::BF16 and
// backend_t::CUDA.
#ifndef EINSUM_IR_B200_CONSTANTS_H
#define EINSUM_IR_B200_CONSTANTS_H

#include <cstdint>

namespace einsum_ir {

typedef enum {
  C = 0,    // left, right, out
  M = 1,    // left, out
  N = 2,    // right, out
  K = 3,    // left, right
  CPX = 4,  // complex dimension (not supported by this backend)
  I = 5,    // left only
  J = 6,    // right only
  UNDEFINED_DIM = 99
} dim_t;

typedef enum {
  SUCCESS = 0,
  COMPILATION_FAILED = 1,
  DIMENSION_ORDERING_FAILED = 2,
  TENSOR_BLOCKING_FAILED = 3,
  NO_DATA_PTR_PROVIDED = 4,
  CALLED_BEFORE_COMPILATION = 5,
  INVALID_ID = 6,
  INVALID_BACKEND = 7,
  INVALID_CPX_DIM = 8,
  INVALID_DTYPE = 9,
  INVALID_KTYPE = 10,
  UNDEFINED_ERROR = 99
} err_t;

typedef enum {
  FP32 = 0,
  FP64 = 1,
  BF16 = 2,  // extension: BF16 storage, FP32 accumulation
  UNDEFINED_DTYPE = 99
} data_t;

typedef enum { REAL_ONLY = 0, BATCH_INNER = 1, BATCH_OUTER = 2, UNDEFINED_CTYPE = 99 } complex_t;

typedef enum {
  ZERO = 0,
  RELU = 1,
  ADD = 2,
  COPY = 3,
  MADD = 4,
  CPX_INT_LOW = 5,
  CPX_ZERO = 6,
  CPX_ADD = 7,
  CPX_MADD = 8,
  CPX_COPY = 9,
  CPX_INT_HIGH = 10,
  CUSTOM_KTYPE = 11,
  BR_MADD = 12,
  PACKED_MADD = 13,
  CPX_PACKED_MADD = 14,
  UNDEFINED_KTYPE = 99
} kernel_t;

typedef enum {
  AUTO = 0,
  SCALAR = 1,
  TPP = 2,
  BLAS = 3,
  TBLIS = 4,
  CUDA = 5,  // extension: this backend
  UNDEFINED_BACKEND = 99
} backend_t;

constexpr int64_t ce_n_bytes(data_t i_dtype) {
  return i_dtype == FP32 ? 4 : i_dtype == FP64 ? 8 : i_dtype == BF16 ? 2 : -1;
}

constexpr bool ce_cpx_op(kernel_t i_ktype) {
  return i_ktype > CPX_INT_LOW && i_ktype < CPX_INT_HIGH;
}

}  // namespace einsum_ir

#endif
