// Dimension analysis shared by all binary contraction backends.
// Rules follow the reference's src/backend/BinaryContraction.cpp (line ranges
// cited per function); the implementation is this backend's own.
#include "BinaryContraction.h"

#include <algorithm>

namespace einsum_ir {
namespace backend {

// Each dim of t2 is matched against the not-yet-matched dims of t0 and t1
// (a match consumes the dim, so repeated ids pair up one by one); the type is
// chosen by where it was found (reference :7-61). The reference erases a t1
// match from the t0 list in the "t1 only" case; here it is consumed from t1,
// which is what the rule intends and identical for unique ids.
void BinaryContraction::dim_types(int64_t i_num_dims_t0, int64_t i_num_dims_t1, int64_t i_num_dims_t2,
                                  int64_t const *i_dim_ids_t0, int64_t const *i_dim_ids_t1,
                                  int64_t const *i_dim_ids_t2, dim_t i_dim_type_t2,
                                  dim_t i_dim_type_t2_t0, dim_t i_dim_type_t2_t1,
                                  dim_t i_dim_type_t2_t0_t1, dim_t *o_dim_types_t2) {
  std::vector<bool> used0(i_num_dims_t0, false), used1(i_num_dims_t1, false);
  auto take = [](int64_t n, int64_t const *ids, std::vector<bool> &used, int64_t id) {
    for (int64_t i = 0; i < n; ++i)
      if (!used[i] && ids[i] == id) {
        used[i] = true;
        return true;
      }
    return false;
  };
  for (int64_t d = 0; d < i_num_dims_t2; ++d) {
    int64_t id = i_dim_ids_t2[d];
    bool in0 = take(i_num_dims_t0, i_dim_ids_t0, used0, id);
    bool in1 = take(i_num_dims_t1, i_dim_ids_t1, used1, id);
    o_dim_types_t2[d] = (in0 && in1) ? i_dim_type_t2_t0_t1
                        : in0        ? i_dim_type_t2_t0
                        : in1        ? i_dim_type_t2_t1
                                     : i_dim_type_t2;
  }
}

void BinaryContraction::dim_types(int64_t i_num_dims_left, int64_t i_num_dims_right,
                                  int64_t i_num_dims_out, int64_t const *i_dim_ids_left,
                                  int64_t const *i_dim_ids_right, int64_t const *i_dim_ids_out,
                                  std::vector<dim_t> *o_dim_types_left,
                                  std::vector<dim_t> *o_dim_types_right,
                                  std::vector<dim_t> *o_dim_types_out) {
  o_dim_types_left->resize(i_num_dims_left);
  o_dim_types_right->resize(i_num_dims_right);
  o_dim_types_out->resize(i_num_dims_out);
  // left vs (right, out): only left -> I, with right -> K, with out -> M, both -> C
  dim_types(i_num_dims_right, i_num_dims_out, i_num_dims_left, i_dim_ids_right, i_dim_ids_out,
            i_dim_ids_left, I, K, M, C, o_dim_types_left->data());
  // right vs (left, out): only right -> J, with left -> K, with out -> N, both -> C
  dim_types(i_num_dims_left, i_num_dims_out, i_num_dims_right, i_dim_ids_left, i_dim_ids_out,
            i_dim_ids_right, J, K, N, C, o_dim_types_right->data());
  // out vs (left, right): with left -> M, with right -> N, both -> C
  dim_types(i_num_dims_left, i_num_dims_right, i_num_dims_out, i_dim_ids_left, i_dim_ids_right,
            i_dim_ids_out, UNDEFINED_DIM, M, N, C, o_dim_types_out->data());
}

int64_t BinaryContraction::filter_dim_ids(int64_t i_num_dims_tensor, dim_t i_dim_type_filter,
                                          dim_t const *i_dim_types_tensor,
                                          int64_t const *i_dim_ids_tensor,
                                          int64_t *o_dim_ids_filtered) {
  int64_t n = 0;
  for (int64_t d = 0; d < i_num_dims_tensor; ++d)
    if (i_dim_types_tensor[d] == i_dim_type_filter) o_dim_ids_filtered[n++] = i_dim_ids_tensor[d];
  return n;
}

void BinaryContraction::dim_types_ids(int64_t i_num_dims_left, int64_t i_num_dims_right,
                                      int64_t i_num_dims_out, int64_t const *i_dim_ids_left,
                                      int64_t const *i_dim_ids_right, int64_t const *i_dim_ids_out,
                                      std::vector<dim_t> *o_dim_types_out,
                                      std::vector<int64_t> *o_dim_ids_c,
                                      std::vector<int64_t> *o_dim_ids_m,
                                      std::vector<int64_t> *o_dim_ids_n,
                                      std::vector<int64_t> *o_dim_ids_k,
                                      std::vector<int64_t> *o_dim_ids_i,
                                      std::vector<int64_t> *o_dim_ids_j) {
  std::vector<dim_t> tl, tr;
  dim_types(i_num_dims_left, i_num_dims_right, i_num_dims_out, i_dim_ids_left, i_dim_ids_right,
            i_dim_ids_out, &tl, &tr, o_dim_types_out);
  auto collect = [](int64_t n, dim_t const *types, int64_t const *ids, dim_t t,
                    std::vector<int64_t> *dst) {
    dst->clear();
    for (int64_t d = 0; d < n; ++d)
      if (types[d] == t) dst->push_back(ids[d]);
  };
  collect(i_num_dims_out, o_dim_types_out->data(), i_dim_ids_out, C, o_dim_ids_c);
  collect(i_num_dims_out, o_dim_types_out->data(), i_dim_ids_out, M, o_dim_ids_m);
  collect(i_num_dims_out, o_dim_types_out->data(), i_dim_ids_out, N, o_dim_ids_n);
  collect(i_num_dims_left, tl.data(), i_dim_ids_left, K, o_dim_ids_k);
  collect(i_num_dims_left, tl.data(), i_dim_ids_left, I, o_dim_ids_i);
  collect(i_num_dims_right, tr.data(), i_dim_ids_right, J, o_dim_ids_j);
}

void BinaryContraction::strides(int64_t i_num_dims, int64_t const *i_dim_ids,
                                std::map<int64_t, int64_t> const *i_dim_sizes,
                                std::map<int64_t, int64_t> *o_strides) {
  o_strides->clear();
  int64_t s = 1;
  for (int64_t d = i_num_dims - 1; d >= 0; --d) {
    int64_t id = i_dim_ids[d];
    int64_t size = i_dim_sizes->at(id);
    o_strides->insert({id, size < 2 ? 0 : s});
    s *= size;
  }
}

void BinaryContraction::init(int64_t i_num_dims_left, int64_t i_num_dims_right, int64_t i_num_dims_out,
                             std::map<int64_t, int64_t> const *i_dim_sizes_inner,
                             std::map<int64_t, int64_t> const *i_dim_sizes_outer_left,
                             std::map<int64_t, int64_t> const *i_dim_sizes_outer_right,
                             std::map<int64_t, int64_t> const *i_dim_sizes_outer_out_aux,
                             std::map<int64_t, int64_t> const *i_dim_sizes_outer_out,
                             int64_t const *i_dim_ids_left, int64_t const *i_dim_ids_right,
                             int64_t const *i_dim_ids_out, data_t i_dtype_left, data_t i_dtype_right,
                             data_t i_dtype_comp, data_t i_dtype_out, kernel_t i_ktype_first_touch,
                             kernel_t i_ktype_main, kernel_t i_ktype_last_touch,
                             int64_t i_num_threads) {
  init(i_num_dims_left, i_num_dims_right, i_num_dims_out, i_dim_sizes_inner, i_dim_sizes_outer_left,
       i_dim_sizes_outer_right, i_dim_sizes_outer_out_aux, i_dim_sizes_outer_out, nullptr,
       i_dim_ids_left, i_dim_ids_right, i_dim_ids_out, nullptr, nullptr, nullptr, i_dtype_left,
       i_dtype_right, i_dtype_comp, i_dtype_out, i_ktype_first_touch, i_ktype_main,
       i_ktype_last_touch, i_num_threads);
}

void BinaryContraction::init(int64_t i_num_dims_left, int64_t i_num_dims_right, int64_t i_num_dims_out,
                             std::map<int64_t, int64_t> const *i_dim_sizes_inner,
                             std::map<int64_t, int64_t> const *i_dim_sizes_outer_left,
                             std::map<int64_t, int64_t> const *i_dim_sizes_outer_right,
                             std::map<int64_t, int64_t> const *i_dim_sizes_outer_out_aux,
                             std::map<int64_t, int64_t> const *i_dim_sizes_outer_out,
                             std::vector<int64_t> const *i_loop_ids_ext, int64_t const *i_dim_ids_left,
                             int64_t const *i_dim_ids_right, int64_t const *i_dim_ids_out,
                             int64_t const *i_dim_ids_permute_left,
                             int64_t const *i_dim_ids_permute_right, MemoryManager *i_memory,
                             data_t i_dtype_left, data_t i_dtype_right, data_t i_dtype_comp,
                             data_t i_dtype_out, kernel_t i_ktype_first_touch, kernel_t i_ktype_main,
                             kernel_t i_ktype_last_touch, int64_t i_num_threads) {
  m_num_dims_left = i_num_dims_left;
  m_num_dims_right = i_num_dims_right;
  m_num_dims_out = i_num_dims_out;
  m_dim_sizes_inner = i_dim_sizes_inner;
  m_dim_sizes_outer_left = i_dim_sizes_outer_left;
  m_dim_sizes_outer_right = i_dim_sizes_outer_right;
  m_dim_sizes_outer_out_aux = i_dim_sizes_outer_out_aux;
  m_dim_sizes_outer_out = i_dim_sizes_outer_out;
  m_loop_ids_ext = i_loop_ids_ext;
  m_dim_ids_left = i_dim_ids_left;
  m_dim_ids_right = i_dim_ids_right;
  m_dim_ids_out = i_dim_ids_out;
  m_dim_ids_permute_left = i_dim_ids_permute_left;
  m_dim_ids_permute_right = i_dim_ids_permute_right;
  m_memory = i_memory;
  m_dtype_left = i_dtype_left;
  m_dtype_right = i_dtype_right;
  m_dtype_comp = i_dtype_comp;
  m_dtype_out = i_dtype_out;
  m_ktype_first_touch = i_ktype_first_touch;
  m_ktype_main = i_ktype_main;
  m_ktype_last_touch = i_ktype_last_touch;
  m_num_threads = i_num_threads;
}

err_t BinaryContraction::compile_base() {
  dim_types_ids(m_num_dims_left, m_num_dims_right, m_num_dims_out, m_dim_ids_left, m_dim_ids_right,
                m_dim_ids_out, &m_dim_types_out, &m_dim_ids_c, &m_dim_ids_m, &m_dim_ids_n,
                &m_dim_ids_k, &m_dim_ids_i, &m_dim_ids_j);
  m_num_dims_c = (int64_t)m_dim_ids_c.size();
  m_num_dims_m = (int64_t)m_dim_ids_m.size();
  m_num_dims_n = (int64_t)m_dim_ids_n.size();
  m_num_dims_k = (int64_t)m_dim_ids_k.size();
  m_num_dims_i = (int64_t)m_dim_ids_i.size();
  m_num_dims_j = (int64_t)m_dim_ids_j.size();
  auto sizes = [this](std::vector<int64_t> const &ids, std::vector<int64_t> *dst) {
    dst->resize(ids.size());
    for (size_t d = 0; d < ids.size(); ++d) (*dst)[d] = m_dim_sizes_inner->at(ids[d]);
  };
  sizes(m_dim_ids_c, &m_sizes_c);
  sizes(m_dim_ids_m, &m_sizes_m);
  sizes(m_dim_ids_n, &m_sizes_n);
  sizes(m_dim_ids_k, &m_sizes_k);
  sizes(m_dim_ids_i, &m_sizes_i);
  sizes(m_dim_ids_j, &m_sizes_j);
  m_dim_types.clear();
  for (int64_t id : m_dim_ids_c) m_dim_types.insert({id, C});
  for (int64_t id : m_dim_ids_m) m_dim_types.insert({id, M});
  for (int64_t id : m_dim_ids_n) m_dim_types.insert({id, N});
  for (int64_t id : m_dim_ids_k) m_dim_types.insert({id, K});
  if (m_loop_ids_ext != nullptr) m_loop_ids_int = *m_loop_ids_ext;
  return SUCCESS;
}

int64_t BinaryContraction::num_ops() {
  int64_t c = 1, m = 1, n = 1, k = 1;
  for (int64_t s : m_sizes_c) c *= s;
  for (int64_t s : m_sizes_m) m *= s;
  for (int64_t s : m_sizes_n) n *= s;
  for (int64_t s : m_sizes_k) k *= s;
  int64_t ops = 2 * c * m * n * k;
  if (m_ktype_main == CPX_MADD) ops *= 2;
  if (m_ktype_first_touch == ZERO || m_ktype_first_touch == CPX_ZERO) ops -= c * m * n;
  return ops;
}

}  // namespace backend
}  // namespace einsum_ir
