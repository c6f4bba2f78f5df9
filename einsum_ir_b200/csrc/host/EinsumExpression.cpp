// Expression-to-tree compilation (rules of the reference's
// src/frontend/EinsumExpression.cpp:141-337) and the ascii parsers
// (src/frontend/EinsumExpressionAscii.cpp:8-303), implemented for this backend.
#include "EinsumExpression.h"

#include <algorithm>
#include <deque>
#include <set>
#include <stdexcept>

namespace einsum_ir {
namespace frontend {

void EinsumExpression::histogram(int64_t i_num_dims, int64_t i_string_size,
                                 int64_t const *i_string_dim_ids, int64_t *o_histogram) {
  std::fill(o_histogram, o_histogram + i_num_dims, 0);
  for (int64_t e = 0; e < i_string_size; ++e) o_histogram[i_string_dim_ids[e]]++;
}

void EinsumExpression::substring_out(int64_t i_num_dims_left, int64_t i_num_dims_right,
                                     int64_t const *i_dim_ids_left, int64_t const *i_dim_ids_right,
                                     int64_t *io_histogram, std::vector<int64_t> &o_substring_out) {
  // the two operands are consumed; a dim survives if it still occurs elsewhere
  for (int64_t d = 0; d < i_num_dims_left; ++d) io_histogram[i_dim_ids_left[d]]--;
  for (int64_t d = 0; d < i_num_dims_right; ++d) io_histogram[i_dim_ids_right[d]]--;
  std::set<int64_t> keep;
  for (int64_t d = 0; d < i_num_dims_left; ++d)
    if (io_histogram[i_dim_ids_left[d]] > 0) keep.insert(i_dim_ids_left[d]);
  for (int64_t d = 0; d < i_num_dims_right; ++d)
    if (io_histogram[i_dim_ids_right[d]] > 0) keep.insert(i_dim_ids_right[d]);
  o_substring_out.assign(keep.begin(), keep.end());
  // the new intermediate tensor uses its dims once
  for (int64_t id : o_substring_out) io_histogram[id]++;
}

void EinsumExpression::unique_tensor_ids(int64_t i_num_conts, int64_t const *i_path,
                                         int64_t *o_path) {
  int64_t next = i_num_conts + 1;
  std::deque<int64_t> live;
  for (int64_t t = 0; t < next; ++t) live.push_back(t);
  for (int64_t c = 0; c < i_num_conts; ++c) {
    int64_t p0 = i_path[2 * c], p1 = i_path[2 * c + 1];
    o_path[2 * c] = live[p0];
    o_path[2 * c + 1] = live[p1];
    live.erase(live.begin() + std::max(p0, p1));
    live.erase(live.begin() + std::min(p0, p1));
    live.push_back(next++);
  }
}

void EinsumExpression::init(int64_t i_num_dims, int64_t const *i_dim_sizes, int64_t i_num_conts,
                            int64_t const *i_string_num_dims, int64_t const *i_string_dim_ids,
                            int64_t const *i_path, complex_t i_ctype_ext, data_t i_dtype,
                            void *const *i_data_ptrs) {
  m_num_dims = i_num_dims;
  m_dim_sizes = i_dim_sizes;
  m_num_conts = i_num_conts;
  m_string_num_dims_ext = i_string_num_dims;
  m_string_dim_ids_ext = i_string_dim_ids;
  m_path_ext = i_path;
  m_ctype_ext = i_ctype_ext;
  m_dtype = i_dtype;
  if (m_dtype_inputs == UNDEFINED_DTYPE) m_dtype_inputs = i_dtype;
  m_data_ptrs = i_data_ptrs;
  m_compiled = false;
}

void EinsumExpression::init(int64_t i_num_dims, int64_t const *i_dim_sizes, int64_t i_num_conts,
                            int64_t const *i_string_num_dims, int64_t const *i_string_dim_ids,
                            int64_t const *i_path, data_t i_dtype, void *const *i_data_ptrs) {
  init(i_num_dims, i_dim_sizes, i_num_conts, i_string_num_dims, i_string_dim_ids, i_path, REAL_ONLY,
       i_dtype, i_data_ptrs);
}

err_t EinsumExpression::compile() {
  // complex trees: the complex dim (size 2) is part of every tensor's string
  // (innermost for BATCH_INNER, outermost for BATCH_OUTER) and the contractions
  // use CPX_ZERO / CPX_MADD (reference: EinsumExpression.cpp:213-330). The root
  // contraction writes the user's layout directly: the GPU kernels take any
  // output strides, so the reference's final batch-outer -> batch-inner permute
  // node is not needed.
  if (m_ctype_ext != REAL_ONLY && m_ctype_ext != BATCH_INNER && m_ctype_ext != BATCH_OUTER)
    return INVALID_CPX_DIM;
  const bool cpx = m_ctype_ext != REAL_ONLY;
  if (m_num_conts < 1) return COMPILATION_FAILED;
  const int64_t n_in = m_num_conts + 1;
  m_path_int.assign(2 * m_num_conts, 0);
  unique_tensor_ids(m_num_conts, m_path_ext, m_path_int.data());
  for (int64_t p : m_path_int)
    if (p < 0 || p >= n_in + m_num_conts - 1) return INVALID_ID;

  m_map_dim_sizes.clear();
  for (int64_t d = 0; d < m_num_dims; ++d) m_map_dim_sizes.insert({d, m_dim_sizes[d]});

  // string of all inputs, then one intermediate string per inner contraction
  int64_t size_in = 0;
  for (int64_t t = 0; t < n_in; ++t) size_in += m_string_num_dims_ext[t];
  const int64_t size_all = size_in + m_string_num_dims_ext[n_in];
  for (int64_t e = 0; e < size_all; ++e)
    if (m_string_dim_ids_ext[e] < 0 || m_string_dim_ids_ext[e] >= m_num_dims) return INVALID_ID;
  m_string_dim_ids_int.assign(m_string_dim_ids_ext, m_string_dim_ids_ext + size_in);
  m_string_num_dims_int.assign(m_string_num_dims_ext, m_string_num_dims_ext + n_in);
  std::vector<int64_t> offsets(n_in + 1, 0);
  for (int64_t t = 1; t <= n_in; ++t) offsets[t] = offsets[t - 1] + m_string_num_dims_int[t - 1];

  std::vector<int64_t> hist(m_num_dims);
  histogram(m_num_dims, size_all, m_string_dim_ids_ext, hist.data());
  for (int64_t c = 0; c + 1 < m_num_conts; ++c) {
    int64_t l = m_path_int[2 * c], r = m_path_int[2 * c + 1];
    std::vector<int64_t> sub;
    std::vector<int64_t> ids_l(m_string_dim_ids_int.begin() + offsets[l],
                               m_string_dim_ids_int.begin() + offsets[l] + m_string_num_dims_int[l]);
    std::vector<int64_t> ids_r(m_string_dim_ids_int.begin() + offsets[r],
                               m_string_dim_ids_int.begin() + offsets[r] + m_string_num_dims_int[r]);
    substring_out((int64_t)ids_l.size(), (int64_t)ids_r.size(), ids_l.data(), ids_r.data(),
                  hist.data(), sub);
    m_string_dim_ids_int.insert(m_string_dim_ids_int.end(), sub.begin(), sub.end());
    m_string_num_dims_int.push_back((int64_t)sub.size());
    offsets.push_back((int64_t)m_string_dim_ids_int.size());
  }
  // root: the user's output string
  int64_t const *root_ids = m_string_dim_ids_ext + size_in;
  m_string_num_dims_int.push_back(m_string_num_dims_ext[n_in]);
  m_string_dim_ids_int.insert(m_string_dim_ids_int.end(), root_ids, root_ids + m_string_num_dims_ext[n_in]);
  offsets.push_back((int64_t)m_string_dim_ids_int.size());

  // nodes: inputs, inner contractions (ZERO + MADD), root (reference :240-313)
  const int64_t n_nodes = n_in + m_num_conts;
  m_nodes.clear();
  m_nodes.resize(n_nodes);
  data_t dt_inner = m_dtype;
  for (int64_t t = 0; t < n_in; ++t)
    m_nodes[t].init(m_string_num_dims_int[t], m_string_dim_ids_int.data() + offsets[t],
                    &m_map_dim_sizes, nullptr, m_dtype_inputs,
                    m_data_ptrs != nullptr ? m_data_ptrs[t] : nullptr, &m_memory);
  for (int64_t c = 0; c < m_num_conts; ++c) {
    int64_t l = m_path_int[2 * c], r = m_path_int[2 * c + 1];
    int64_t out = n_in + c;
    bool root = c + 1 == m_num_conts;
    m_nodes[out].init(m_string_num_dims_int[out], m_string_dim_ids_int.data() + offsets[out],
                      &m_map_dim_sizes, nullptr, nullptr, nullptr, nullptr, dt_inner, nullptr,
                      root && m_data_ptrs != nullptr ? m_data_ptrs[n_in] : nullptr,
                      cpx ? CPX_ZERO : ZERO, cpx ? CPX_MADD : MADD, UNDEFINED_KTYPE, &m_nodes[l],
                      &m_nodes[r], &m_memory, 1);
  }
  for (auto &n : m_nodes) n.m_compute = m_compute;
  err_t err = m_nodes.back().compile();
  if (m_stream != nullptr) m_nodes.back().set_stream(m_stream);
  m_compiled = true;
  return err;
}

err_t EinsumExpression::store_and_lock_data(int64_t i_tensor_id) {
  if (!m_compiled) return CALLED_BEFORE_COMPILATION;
  if (i_tensor_id < 0 || i_tensor_id >= m_num_conts + 1) return INVALID_ID;
  return m_nodes[i_tensor_id].store_and_lock_data();
}

err_t EinsumExpression::unlock_data(int64_t i_tensor_id) {
  if (!m_compiled) return CALLED_BEFORE_COMPILATION;
  if (i_tensor_id < 0 || i_tensor_id >= m_num_conts + 1) return INVALID_ID;
  return m_nodes[i_tensor_id].unlock_data();
}

int EinsumExpression::eval() {
  if (m_nodes.empty()) return CALLED_BEFORE_COMPILATION;
  return m_nodes.back().eval();
}

int64_t EinsumExpression::num_ops() { return m_nodes.empty() ? 0 : m_nodes.back().num_ops(true); }

void EinsumExpression::set_stream(void *i_stream) {
  m_stream = i_stream;  // applied to the nodes now and at every compile
  if (!m_nodes.empty()) m_nodes.back().set_stream(i_stream);
}

void EinsumExpression::set_data_ptrs(void *const *i_data_ptrs) {
  const int64_t n_in = m_num_conts + 1;
  for (int64_t t = 0; t < n_in; ++t) m_nodes[t].m_data_ptr_ext = i_data_ptrs[t];
  m_nodes.back().m_data_ptr_ext = i_data_ptrs[n_in];
}

// ------------------------------------------------------------------ ascii parsers
void EinsumExpressionAscii::split_string(std::string const &i_input, std::string const &i_separation,
                                         std::vector<std::string> &o_output) {
  size_t pos = 0;
  while (true) {
    size_t hit = i_input.find(i_separation, pos);
    if (hit == std::string::npos) {
      if (pos < i_input.size()) o_output.push_back(i_input.substr(pos));
      return;
    }
    o_output.push_back(i_input.substr(pos, hit - pos));
    pos = hit + i_separation.size();
  }
}

static std::string strip_spaces(std::string s) {
  s.erase(std::remove(s.begin(), s.end(), ' '), s.end());
  return s;
}

void EinsumExpressionAscii::schar_to_standard(std::string const &i_expr_string,
                                              std::string &o_expr_string) {
  std::string e = strip_spaces(i_expr_string);
  std::vector<std::string> sides, ins;
  split_string(e, "->", sides);
  if (sides.empty()) sides.push_back("");
  if (sides.size() == 1) sides.push_back("");
  split_string(sides[0], ",", ins);
  auto bracket = [](std::string const &t) {
    std::string s = "[";
    for (size_t i = 0; i < t.size(); ++i) {
      s += t[i];
      if (i + 1 < t.size()) s += ",";
    }
    return s + "]";
  };
  o_expr_string.clear();
  for (size_t t = 0; t < ins.size(); ++t) {
    o_expr_string += bracket(ins[t]);
    if (t + 1 < ins.size()) o_expr_string += ",";
  }
  o_expr_string += "->" + bracket(sides[1]);
}

// numbers compare numerically, anything else lexicographically (the reference's
// comparator: std::stoi on both names, falling back to string order)
static bool dim_name_less(std::string const &a, std::string const &b) {
  try {
    return std::stoi(a) < std::stoi(b);
  } catch (...) {
    return a < b;
  }
}

void EinsumExpressionAscii::parse_tensors(std::string const &i_expr_string,
                                          std::vector<std::string> &o_tensors) {
  o_tensors.clear();
  std::string e = strip_spaces(i_expr_string);
  if (e.size() >= 2) e = e.substr(1, e.size() - 2);  // outer brackets
  std::vector<std::string> sides;
  split_string(e, "]->[", sides);
  if (sides.empty()) sides.push_back("");
  if (sides.size() == 1) sides.push_back("");
  split_string(sides[0], "],[", o_tensors);
  o_tensors.push_back(sides[1]);
}

void EinsumExpressionAscii::parse_dim_sizes(std::string const &i_dim_sizes_string,
                                            std::vector<int64_t> &o_dim_sizes) {
  o_dim_sizes.clear();
  std::vector<std::string> parts;
  split_string(strip_spaces(i_dim_sizes_string), ",", parts);
  for (auto const &p : parts) o_dim_sizes.push_back(std::stoll(p));
}

void EinsumExpressionAscii::parse_path(std::string const &i_expr_string, std::vector<int64_t> &o_path) {
  o_path.clear();
  std::string e;
  for (char ch : i_expr_string)
    if (ch != ' ' && ch != '(' && ch != ')') e += ch;
  std::vector<std::string> parts;
  split_string(e, ",", parts);
  for (auto const &p : parts) o_path.push_back(std::stoll(p));
}

void EinsumExpressionAscii::parse_dim_ids(std::string const &i_expr_string,
                                          std::map<std::string, int64_t> &o_map_dim_name_to_id) {
  o_map_dim_name_to_id.clear();
  std::vector<std::string> tensors;
  parse_tensors(i_expr_string, tensors);
  std::set<std::string> names;
  for (auto const &t : tensors) {
    std::vector<std::string> dims;
    split_string(t, ",", dims);
    names.insert(dims.begin(), dims.end());
  }
  std::vector<std::string> sorted(names.begin(), names.end());
  std::sort(sorted.begin(), sorted.end(), dim_name_less);
  for (size_t i = 0; i < sorted.size(); ++i) o_map_dim_name_to_id.insert({sorted[i], (int64_t)i});
}

void EinsumExpressionAscii::standard_to_schar(std::string const &i_expr_string,
                                              std::string &o_expr_string) {
  std::map<std::string, int64_t> ids;
  parse_dim_ids(i_expr_string, ids);
  std::vector<std::string> tensors;
  parse_tensors(i_expr_string, tensors);
  auto to_char = [&](int64_t id) -> std::string {
    if (ids.size() <= 52) return std::string(1, (char)(id < 26 ? 'A' + id : 'a' + id - 26));
    uint32_t cp = (uint32_t)(id + 161);  // UTF-8 encode code point 161 + id
    std::string s;
    if (cp < 0x800) {
      s += (char)(0xC0 | (cp >> 6));
      s += (char)(0x80 | (cp & 0x3F));
    } else {
      s += (char)(0xE0 | (cp >> 12));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    }
    return s;
  };
  o_expr_string.clear();
  for (size_t t = 0; t < tensors.size(); ++t) {
    std::vector<std::string> dims;
    split_string(tensors[t], ",", dims);
    for (auto const &d : dims) o_expr_string += to_char(ids.at(d));
    if (t + 2 < tensors.size()) o_expr_string += ",";
    else if (t + 2 == tensors.size()) o_expr_string += "->";
  }
}

void EinsumExpressionAscii::parse_ctype(std::string const &i_ctype_string, complex_t &o_ctype) {
  // complex data types keep the complex dim innermost (interleaved)
  if (i_ctype_string == "FP32" || i_ctype_string == "FP64" || i_ctype_string == "BF16") o_ctype = REAL_ONLY;
  else if (i_ctype_string == "CPX_FP32" || i_ctype_string == "CPX_FP64") o_ctype = BATCH_INNER;
  else o_ctype = UNDEFINED_CTYPE;
}

void EinsumExpressionAscii::parse_dtype(std::string const &i_dtype_string, data_t &o_dtype) {
  if (i_dtype_string == "FP32" || i_dtype_string == "CPX_FP32") o_dtype = FP32;
  else if (i_dtype_string == "FP64" || i_dtype_string == "CPX_FP64") o_dtype = FP64;
  else if (i_dtype_string == "BF16") o_dtype = BF16;
  else o_dtype = UNDEFINED_DTYPE;
}

}  // namespace frontend
}  // namespace einsum_ir
