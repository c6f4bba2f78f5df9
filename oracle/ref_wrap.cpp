// C wrappers around the reference's structural host functions, compiled from
// the reference sources where they lie (see oracle/ref.mk). TEST
// INFRASTRUCTURE ONLY: used by tests/ to check this backend's host logic
// against the reference itself. Only functions that need no libxsmm are
// wrapped (dim typing, the swap rule, expression helpers, ascii parsers).
#include <cstring>
#include <map>
#include <string>
#include <vector>
#include "backend/BinaryContraction.h"
#include "backend/BinaryPrimitives.h"
#include "frontend/EinsumExpression.h"
#include "frontend/EinsumExpressionAscii.h"
#include "frontend/EinsumTreeAscii.h"

using einsum_ir::backend::BinaryContraction;
using einsum_ir::backend::BinaryPrimitives;
using einsum_ir::frontend::EinsumExpression;
using einsum_ir::frontend::EinsumExpressionAscii;
using einsum_ir::frontend::EinsumTreeAscii;

extern "C" {

void ref_dim_types(int64_t nl, int64_t nr, int64_t no, const int64_t *l, const int64_t *r,
                   const int64_t *o, int32_t *tl, int32_t *tr, int32_t *to) {
  std::vector<einsum_ir::dim_t> a, b, c;
  BinaryContraction::dim_types(nl, nr, no, l, r, o, &a, &b, &c);
  for (int64_t i = 0; i < nl; ++i) tl[i] = a[i];
  for (int64_t i = 0; i < nr; ++i) tr[i] = b[i];
  for (int64_t i = 0; i < no; ++i) to[i] = c[i];
}

int ref_swap_inputs(int64_t nl, int64_t nr, int64_t no, const int64_t *l, const int64_t *r,
                    const int64_t *o) {
  return BinaryPrimitives::swap_inputs(nl, nr, no, l, r, o) ? 1 : 0;
}

void ref_strides(int64_t n, const int64_t *ids, const int64_t *sizes_by_pos, int64_t *strides_by_pos) {
  std::map<int64_t, int64_t> sz, st;
  for (int64_t i = 0; i < n; ++i) sz[ids[i]] = sizes_by_pos[i];
  BinaryContraction::strides(n, ids, &sz, &st);
  for (int64_t i = 0; i < n; ++i) strides_by_pos[i] = st[ids[i]];
}

void ref_unique_tensor_ids(int64_t nconts, const int64_t *path, int64_t *out) {
  EinsumExpression::unique_tensor_ids(nconts, path, out);
}

// returns the number of output dims written to out (capacity cap)
int64_t ref_substring_out(int64_t nl, int64_t nr, const int64_t *l, const int64_t *r, int64_t *hist,
                          int64_t *out, int64_t cap) {
  std::vector<int64_t> s;
  EinsumExpression::substring_out(nl, nr, l, r, hist, s);
  for (size_t i = 0; i < s.size() && (int64_t)i < cap; ++i) out[i] = s[i];
  return (int64_t)s.size();
}

// dim name -> id for a standard-format expression; writes "name:id;" pairs
int64_t ref_parse_dim_ids(const char *expr, char *out, int64_t cap) {
  std::map<std::string, int64_t> m;
  EinsumExpressionAscii::parse_dim_ids(expr, m);
  std::string s;
  for (auto const &kv : m) s += kv.first + ":" + std::to_string(kv.second) + ";";
  std::strncpy(out, s.c_str(), (size_t)cap);
  return (int64_t)s.size();
}

int64_t ref_schar_to_standard(const char *expr, char *out, int64_t cap) {
  std::string s;
  EinsumExpressionAscii::schar_to_standard(expr, s);
  std::strncpy(out, s.c_str(), (size_t)cap);
  return (int64_t)s.size();
}

// einsum tree string -> "ids:children;" per node (post order) then "|id=size,"
// for the dimension sizes; returns -1 if the reference parser rejects the tree
int64_t ref_parse_tree(const char *tree, const char *sizes, char *out, int64_t cap) {
  std::string t(tree);
  int64_t n = EinsumTreeAscii::count_nodes(t);
  std::vector<std::vector<int64_t>> ids(n), ch(n);
  int64_t next = 0;
  if (EinsumTreeAscii::parse_tree(t, ids, ch, next) != einsum_ir::SUCCESS || next != n) return -1;
  std::map<int64_t, int64_t> sz;
  EinsumTreeAscii::parse_dim_size(sizes, ids, sz);
  std::string s;
  for (int64_t i = 0; i < n; ++i) {
    for (auto x : ids[i]) s += std::to_string(x) + ",";
    s += ":";
    for (auto x : ch[i]) s += std::to_string(x) + ",";
    s += ";";
  }
  s += "|";
  for (auto const &kv : sz) s += std::to_string(kv.first) + "=" + std::to_string(kv.second) + ",";
  std::strncpy(out, s.c_str(), (size_t)cap);
  return (int64_t)s.size();
}

}  // extern "C"
