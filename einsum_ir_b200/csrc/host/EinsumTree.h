// EinsumTree / EinsumTreeAscii: a pre-optimised contraction tree given as
// nodes (dimension ids + children) instead of an expression and a path, as in
// the reference's src/frontend/EinsumTree.h:12-73 and EinsumTreeAscii.h.
//
// Tree strings: a leaf is a comma-separated list of dimension ids; an inner
// node is "[left],[right]->[out]" (binary contraction) or "[child]->[out]"
// (permute). Nodes are numbered in post order (children before parents, the
// root last), e.g. "[[3,0]->[0,3]],[[3,2,4],[1,4,2]->[1,2,3]]->[0,1,2]" has
// nodes {3,0} {0,3} {3,2,4} {1,4,2} {1,2,3} {0,1,2} with children
// {} {0} {} {} {2,3} {1,4}.
#ifndef EINSUM_IR_B200_EINSUM_TREE_H
#define EINSUM_IR_B200_EINSUM_TREE_H

#include <map>
#include <string>
#include <vector>
#include "EinsumNode.h"
#include "MemoryManager.h"
#include "constants.h"

namespace einsum_ir {
namespace frontend {

class EinsumTree {
 public:
  //! nodes of the tree (post order, root last)
  std::vector<backend::EinsumNode> m_nodes;
  //! dimension ids and children of every node (borrowed)
  std::vector<std::vector<int64_t>> *m_dim_ids = nullptr;
  std::vector<std::vector<int64_t>> *m_children = nullptr;
  //! data pointers of every node: leaves and root external, inner nodes nullptr
  void *const *m_data_ptrs = nullptr;
  backend::MemoryManager m_memory;
  data_t m_dtype = UNDEFINED_DTYPE;
  std::map<int64_t, int64_t> *m_map_dim_sizes = nullptr;

  void init(std::vector<std::vector<int64_t>> *i_dim_ids,
            std::vector<std::vector<int64_t>> *i_children,
            std::map<int64_t, int64_t> *i_map_dim_sizes, data_t i_dtype, void *const *i_data_ptrs);
  err_t compile();
  //! enqueues the evaluation on the tree's stream; returns the first error status
  //! (the reference's eval returns nothing)
  int eval();
  int64_t num_ops();

  //! extensions of this backend (call before compile): storage type of the
  //! leaves (BF16 leaves with FP32 inner nodes), compute type, stream
  void set_input_dtype(data_t i_dtype) { m_dtype_inputs = i_dtype; }
  void set_compute_type(int32_t i_comp) { m_compute = i_comp; }
  void set_stream(void *i_stream);

 private:
  data_t m_dtype_inputs = UNDEFINED_DTYPE;
  int32_t m_compute = 0;
  void *m_stream = nullptr;
};

class EinsumTreeAscii {
 public:
  static void split_string(std::string const &i_input, std::string const &i_separation,
                           std::vector<std::string> &o_output);
  //! number of nodes of a tree string
  static int64_t count_nodes(std::string const &i_string_tree);
  //! parses a (sub)tree into o_dim_ids / o_children (sized by count_nodes)
  //! starting at node id io_node_id, which ends one past the subtree's root
  static err_t parse_tree(std::string const &i_string_tree, std::vector<std::vector<int64_t>> &o_dim_ids,
                          std::vector<std::vector<int64_t>> &o_children, int64_t &io_node_id);
  static void parse_vector(std::string const &i_string_vector, std::vector<int64_t> &o_int_vector);
  //! sizes in ascending order of the dimension ids used by the tree
  static void parse_dim_size(std::string const &i_string_sizes,
                             std::vector<std::vector<int64_t>> const &i_dim_ids,
                             std::map<int64_t, int64_t> &o_map_dim_sizes);
  //! "[left],[right]->[out]" or "[child]->[out]" -> the bracket contents
  static err_t split_outer_operation(std::string const &i_string_tree, std::string &o_left_tree,
                                     std::string &o_right_tree, std::string &o_out_tree);
};

}  // namespace frontend
}  // namespace einsum_ir

#endif
