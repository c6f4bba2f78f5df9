#include "BinaryPrimitives.h"

#include <algorithm>
#include <vector>
#include "BinaryContraction.h"

namespace einsum_ir {
namespace backend {

bool BinaryPrimitives::swap_inputs(int64_t i_num_dims_left, int64_t i_num_dims_right,
                                   int64_t i_num_dims_out, int64_t const *i_dim_ids_left,
                                   int64_t const *i_dim_ids_right, int64_t const *i_dim_ids_out) {
  std::vector<dim_t> tl, tr, to;
  BinaryContraction::dim_types(i_num_dims_left, i_num_dims_right, i_num_dims_out, i_dim_ids_left,
                               i_dim_ids_right, i_dim_ids_out, &tl, &tr, &to);
  if (to.empty()) return false;
  if (to.back() == N) return true;
  if (to.back() != C) return false;
  // fastest output dim is C: the first M or N dim further out decides
  for (int64_t d = (int64_t)to.size() - 1; d >= 0; --d) {
    if (to[d] == M) return false;
    if (to[d] == N) return true;
  }
  return false;
}

err_t BinaryPrimitives::reorder(int64_t i_num_dims_left, int64_t i_num_dims_right,
                                int64_t i_num_dims_out, std::map<int64_t, int64_t> const *,
                                bool i_left_free, bool i_right_free, int64_t *io_dim_ids_left,
                                int64_t *io_dim_ids_right, int64_t const *i_dim_ids_out) {
  if (!i_left_free && !i_right_free) return SUCCESS;
  std::vector<dim_t> tl, tr, to;
  BinaryContraction::dim_types(i_num_dims_left, i_num_dims_right, i_num_dims_out, io_dim_ids_left,
                               io_dim_ids_right, i_dim_ids_out, &tl, &tr, &to);
  // K order: taken from an operand whose layout is fixed, else ascending ids
  std::vector<int64_t> k_order;
  if (!i_left_free) {
    for (int64_t d = 0; d < i_num_dims_left; ++d)
      if (tl[d] == K) k_order.push_back(io_dim_ids_left[d]);
  } else if (!i_right_free) {
    for (int64_t d = 0; d < i_num_dims_right; ++d)
      if (tr[d] == K) k_order.push_back(io_dim_ids_right[d]);
  } else {
    for (int64_t d = 0; d < i_num_dims_left; ++d)
      if (tl[d] == K) k_order.push_back(io_dim_ids_left[d]);
    std::sort(k_order.begin(), k_order.end());
  }
  auto relayout = [&](int64_t n, int64_t *ids, std::vector<dim_t> const &types) {
    std::vector<int64_t> out;
    for (int64_t d = 0; d < i_num_dims_out; ++d)  // C dims, output order
      for (int64_t e = 0; e < n; ++e)
        if (ids[e] == i_dim_ids_out[d] && types[e] == C) out.push_back(ids[e]);
    for (int64_t d = 0; d < i_num_dims_out; ++d)  // M / N dims, output order
      for (int64_t e = 0; e < n; ++e)
        if (ids[e] == i_dim_ids_out[d] && (types[e] == M || types[e] == N)) out.push_back(ids[e]);
    for (int64_t e = 0; e < n; ++e)  // one-sided dims (kept, before K)
      if (types[e] == I || types[e] == J) out.push_back(ids[e]);
    for (int64_t k : k_order) out.push_back(k);  // K dims, shared order, innermost
    if ((int64_t)out.size() != n) return false;
    std::copy(out.begin(), out.end(), ids);
    return true;
  };
  if (i_left_free && !relayout(i_num_dims_left, io_dim_ids_left, tl)) return DIMENSION_ORDERING_FAILED;
  if (i_right_free && !relayout(i_num_dims_right, io_dim_ids_right, tr)) return DIMENSION_ORDERING_FAILED;
  return SUCCESS;
}

}  // namespace backend
}  // namespace einsum_ir
