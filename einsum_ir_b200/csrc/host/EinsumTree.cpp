// EinsumTree / EinsumTreeAscii (reference: src/frontend/EinsumTree.cpp:5-102,
// src/frontend/EinsumTreeAscii.cpp:5-199). Node kinds follow the reference:
// no children = leaf (external data), one child = permute node, two children
// = binary contraction with ZERO first touch and MADD main kernel.
#include "EinsumTree.h"

#include <algorithm>
#include <set>

namespace einsum_ir {
namespace frontend {

void EinsumTree::init(std::vector<std::vector<int64_t>> *i_dim_ids,
                      std::vector<std::vector<int64_t>> *i_children,
                      std::map<int64_t, int64_t> *i_map_dim_sizes, data_t i_dtype,
                      void *const *i_data_ptrs) {
  m_dim_ids = i_dim_ids;
  m_children = i_children;
  m_map_dim_sizes = i_map_dim_sizes;
  m_dtype = i_dtype;
  m_data_ptrs = i_data_ptrs;
}

err_t EinsumTree::compile() {
  if (m_dim_ids == nullptr || m_children == nullptr || m_map_dim_sizes == nullptr ||
      m_data_ptrs == nullptr || m_children->empty() || m_dim_ids->size() != m_children->size())
    return COMPILATION_FAILED;
  const size_t n = m_children->size();
  // children come before their parents (post order)
  for (size_t id = 0; id < n; ++id) {
    auto const &ch = (*m_children)[id];
    if (ch.size() > 2) return COMPILATION_FAILED;
    for (int64_t c : ch)
      if (c < 0 || (size_t)c >= id) return INVALID_ID;
  }
  const data_t dt_leaf = m_dtype_inputs == UNDEFINED_DTYPE ? m_dtype : m_dtype_inputs;
  m_nodes.clear();
  m_nodes.resize(n);
  for (size_t id = 0; id < n; ++id) {
    auto const &ch = (*m_children)[id];
    auto const &ids = (*m_dim_ids)[id];
    backend::EinsumNode &node = m_nodes[id];
    void *ptr = m_data_ptrs[id];
    if (ch.empty()) {
      node.init((int64_t)ids.size(), ids.data(), m_map_dim_sizes, nullptr, dt_leaf, ptr, &m_memory);
    } else if (ch.size() == 1) {
      // a permute of a leaf keeps the leaf's storage type
      data_t dt = (*m_children)[ch[0]].empty() ? dt_leaf : m_dtype;
      node.init((int64_t)ids.size(), ids.data(), m_map_dim_sizes, nullptr, dt, ptr, &m_nodes[ch[0]],
                &m_memory, 1);
    } else {
      node.init((int64_t)ids.size(), ids.data(), m_map_dim_sizes, nullptr, nullptr, nullptr, nullptr,
                m_dtype, nullptr, ptr, ZERO, MADD, UNDEFINED_KTYPE, &m_nodes[ch[0]], &m_nodes[ch[1]],
                &m_memory, 1);
    }
    node.m_compute = m_compute;
  }
  err_t err = m_nodes.back().compile();
  if (m_stream != nullptr) m_nodes.back().set_stream(m_stream);
  return err;
}

int EinsumTree::eval() {
  if (m_nodes.empty()) return CALLED_BEFORE_COMPILATION;
  return m_nodes.back().eval();
}

int64_t EinsumTree::num_ops() { return m_nodes.empty() ? 0 : m_nodes.back().num_ops(true); }

void EinsumTree::set_stream(void *i_stream) {
  m_stream = i_stream;
  if (!m_nodes.empty()) m_nodes.back().set_stream(i_stream);
}

// ------------------------------------------------------------------ ascii parsers
void EinsumTreeAscii::split_string(std::string const &i_input, std::string const &i_separation,
                                   std::vector<std::string> &o_output) {
  size_t pos = 0;
  while (pos < i_input.size()) {
    size_t hit = i_input.find(i_separation, pos);
    if (hit == std::string::npos) {
      o_output.push_back(i_input.substr(pos));
      return;
    }
    o_output.push_back(i_input.substr(pos, hit - pos));
    pos = hit + i_separation.size();
  }
}

int64_t EinsumTreeAscii::count_nodes(std::string const &i_string_tree) {
  // one node per "],[" (a second child) and per "]->[" (an inner node), plus
  // the first leaf
  int64_t count = 1;
  for (size_t i = 0; i + 3 < i_string_tree.size(); ++i) {
    if (i_string_tree.compare(i, 3, "],[") == 0) ++count;
    if (i_string_tree.compare(i, 4, "]->[") == 0) ++count;
  }
  return count;
}

void EinsumTreeAscii::parse_vector(std::string const &i_string_vector,
                                   std::vector<int64_t> &o_int_vector) {
  std::string s = i_string_vector;
  s.erase(std::remove(s.begin(), s.end(), ' '), s.end());
  std::vector<std::string> parts;
  split_string(s, ",", parts);
  o_int_vector.clear();
  for (auto const &p : parts) o_int_vector.push_back(std::stoll(p));
}

void EinsumTreeAscii::parse_dim_size(std::string const &i_string_sizes,
                                     std::vector<std::vector<int64_t>> const &i_dim_ids,
                                     std::map<int64_t, int64_t> &o_map_dim_sizes) {
  std::vector<int64_t> sizes;
  parse_vector(i_string_sizes, sizes);
  std::set<int64_t> ids;  // ascending
  for (auto const &t : i_dim_ids) ids.insert(t.begin(), t.end());
  o_map_dim_sizes.clear();
  size_t k = 0;
  for (int64_t id : ids) {
    if (k >= sizes.size()) break;
    o_map_dim_sizes[id] = sizes[k++];
  }
}

err_t EinsumTreeAscii::split_outer_operation(std::string const &i_string_tree, std::string &o_left_tree,
                                             std::string &o_right_tree, std::string &o_out_tree) {
  // top level (bracket depth 0): the last ',' before the '->', then the '->'
  int depth = 0;
  size_t comma = std::string::npos, arrow = std::string::npos;
  for (size_t i = 0; i < i_string_tree.size(); ++i) {
    char c = i_string_tree[i];
    if (c == '[') ++depth;
    if (c == ']') --depth;
    if (depth != 0) continue;
    if (c == ',') comma = i;
    if (c == '-') {
      arrow = i;
      break;
    }
  }
  // pieces are "[...]": drop the enclosing brackets
  auto inner = [&](size_t b, size_t e) -> std::string {
    if (e <= b + 1 || i_string_tree[b] != '[' || i_string_tree[e - 1] != ']') return std::string();
    return i_string_tree.substr(b + 1, e - b - 2);
  };
  if (arrow == std::string::npos || arrow + 2 >= i_string_tree.size() ||
      i_string_tree[arrow + 1] != '>')
    return COMPILATION_FAILED;
  o_out_tree = inner(arrow + 2, i_string_tree.size());
  if (comma != std::string::npos && comma != 0) {
    o_left_tree = inner(0, comma);
    o_right_tree = inner(comma + 1, arrow);
  } else {
    o_left_tree = inner(0, arrow);
    o_right_tree.clear();
  }
  if (o_left_tree.empty() || o_out_tree.empty()) return COMPILATION_FAILED;
  return SUCCESS;
}

err_t EinsumTreeAscii::parse_tree(std::string const &i_string_tree,
                                  std::vector<std::vector<int64_t>> &o_dim_ids,
                                  std::vector<std::vector<int64_t>> &o_children, int64_t &io_node_id) {
  if (io_node_id < 0 || (size_t)io_node_id >= o_dim_ids.size() || o_children.size() < o_dim_ids.size())
    return INVALID_ID;
  if (i_string_tree.empty()) return COMPILATION_FAILED;
  if (i_string_tree[0] != '[') {  // leaf
    try {
      parse_vector(i_string_tree, o_dim_ids[io_node_id]);
    } catch (...) {
      return COMPILATION_FAILED;
    }
    ++io_node_id;
    return SUCCESS;
  }
  std::string left, right, out;
  err_t err = split_outer_operation(i_string_tree, left, right, out);
  if (err != SUCCESS) return err;
  err = parse_tree(left, o_dim_ids, o_children, io_node_id);
  if (err != SUCCESS) return err;
  const int64_t left_id = io_node_id - 1;
  int64_t right_id = -1;
  if (!right.empty()) {
    err = parse_tree(right, o_dim_ids, o_children, io_node_id);
    if (err != SUCCESS) return err;
    right_id = io_node_id - 1;
  }
  if ((size_t)io_node_id >= o_dim_ids.size()) return INVALID_ID;
  o_children[io_node_id].push_back(left_id);
  if (right_id >= 0) o_children[io_node_id].push_back(right_id);
  try {
    parse_vector(out, o_dim_ids[io_node_id]);
  } catch (...) {
    return COMPILATION_FAILED;
  }
  ++io_node_id;
  return SUCCESS;
}

}  // namespace frontend
}  // namespace einsum_ir
