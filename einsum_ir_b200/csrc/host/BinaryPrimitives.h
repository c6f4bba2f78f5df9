// Operand-order decisions for binary contractions in a tree.
//
// swap_inputs follows the reference rule (src/backend/BinaryPrimitives.cpp:87-134):
// the operand holding the output's fastest dim becomes "left" (its dims are M,
// the output rows of a tile), so the tensor-core epilogue writes the output
// coalesced along M.
//
// reorder is this backend's layout policy (the reference's TPP policy
// BC_BM_BK_BI_KB_MB_CB, :833-1117 / :1713-1768, targets CPU GEMM leaves). Only
// operands that are intermediate results of the tree are reordered: their
// layout is free (the child contraction writes it directly), while reordering
// a user input would cost a permute. An intermediate operand is laid out as
//   [C dims][its M or N dims, in output order][K dims]
// with the K dims in the order of the other operand (its K order if that one
// is a user input, ascending ids otherwise), so both operands are K-major
// with the same innermost K dim and the tensor-core path needs no pre-permute.
#ifndef EINSUM_IR_B200_BINARY_PRIMITIVES_H
#define EINSUM_IR_B200_BINARY_PRIMITIVES_H

#include <cstdint>
#include <map>
#include "constants.h"

namespace einsum_ir {
namespace backend {

class BinaryPrimitives {
 public:
  static bool swap_inputs(int64_t i_num_dims_left, int64_t i_num_dims_right, int64_t i_num_dims_out,
                          int64_t const *i_dim_ids_left, int64_t const *i_dim_ids_right,
                          int64_t const *i_dim_ids_out);

  //! reorders the dims of the left / right operands in place where allowed
  static err_t reorder(int64_t i_num_dims_left, int64_t i_num_dims_right, int64_t i_num_dims_out,
                       std::map<int64_t, int64_t> const *i_dim_sizes, bool i_left_free,
                       bool i_right_free, int64_t *io_dim_ids_left, int64_t *io_dim_ids_right,
                       int64_t const *i_dim_ids_out);
};

}  // namespace backend
}  // namespace einsum_ir

#endif
