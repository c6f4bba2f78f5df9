// Node of an einsum contraction tree (interface of the reference's
// backend::EinsumNode, src/backend/EinsumNode.h:16-251).
//
// A node is an input tensor (no children), a permute of its child (one child)
// or a binary contraction of two children. compile() decides operand order
// (swap_inputs), intermediate layouts (reorder), creates the contraction and
// permute plans, and plans the device arena; eval() enqueues the children,
// then the node's permute / contraction, on the tree's CUDA stream. All data
// pointers are device pointers.
#ifndef EINSUM_IR_B200_EINSUM_NODE_H
#define EINSUM_IR_B200_EINSUM_NODE_H

#include <map>
#include <vector>
#include "BinaryContraction.h"
#include "MemoryManager.h"
#include "Unary.h"
#include "constants.h"

namespace einsum_ir {
namespace backend {

class EinsumNode {
 public:
  data_t m_dtype = UNDEFINED_DTYPE;
  kernel_t m_ktype_first_touch = UNDEFINED_KTYPE;
  kernel_t m_ktype_main = UNDEFINED_KTYPE;
  kernel_t m_ktype_last_touch = UNDEFINED_KTYPE;
  int64_t m_size = 0;
  int64_t m_num_dims = 0;
  int64_t const *m_dim_ids_ext = nullptr;
  std::vector<int64_t> m_dim_ids_int;
  std::map<int64_t, int64_t> const *m_dim_sizes_inner = nullptr;
  std::map<int64_t, int64_t> const *m_dim_sizes_aux_outer = nullptr;
  std::map<int64_t, int64_t> const *m_dim_sizes_outer = nullptr;
  std::vector<EinsumNode *> m_children;
  void *m_data_ptr_int = nullptr;
  void *m_data_ptr_ext = nullptr;
  void *m_data_ptr_active = nullptr;
  void *m_data_ptr_aux_int = nullptr;
  void *m_data_ptr_aux_ext = nullptr;
  std::map<int64_t, int64_t> const *m_offsets_aux_ext = nullptr;
  std::map<int64_t, int64_t> const *m_offsets_ext = nullptr;
  int64_t m_offset_aux_bytes = 0;
  int64_t m_offset_bytes = 0;
  bool m_reorder_dims = true;
  bool m_pack_inputs = false;
  backend_t m_btype_unary = UNDEFINED_BACKEND;
  backend_t m_btype_binary = UNDEFINED_BACKEND;
  Unary *m_unary = nullptr;
  BinaryContraction *m_cont = nullptr;
  MemoryManager *m_memory = nullptr;
  int64_t m_mem_id = 0;
  int64_t m_count_mem_users = 0;
  int64_t m_active_mem_users = 0;
  int64_t m_req_mem = 0;
  int64_t m_mem_subtree = 0;
  std::vector<int64_t> m_exec_order;
  int64_t m_num_ops_node = 0;
  int64_t m_num_ops_children = 0;
  int64_t m_num_tasks_intra_op = 1;
  bool m_compiled = false;
  bool m_data_locked = false;
  int64_t m_num_threads = 1;

  //! extensions of this backend: compute type (EIR_COMPUTE_*) and stream
  int32_t m_compute = 0;
  void *m_stream = nullptr;

  ~EinsumNode();

  //! input node
  void init(int64_t i_num_dims, int64_t const *i_dim_ids,
            std::map<int64_t, int64_t> const *i_dim_sizes_inner,
            std::map<int64_t, int64_t> const *i_dim_sizes_outer, data_t i_dtype, void *i_data_ptr,
            MemoryManager *i_memory);

  //! node with a single child (permute)
  void init(int64_t i_num_dims, int64_t const *i_dim_ids,
            std::map<int64_t, int64_t> const *i_dim_sizes_inner,
            std::map<int64_t, int64_t> const *i_dim_sizes_outer, data_t i_dtype, void *i_data_ptr,
            EinsumNode *i_child, MemoryManager *i_memory, int64_t i_num_threads);

  //! node with two children (binary contraction)
  void init(int64_t i_num_dims, int64_t const *i_dim_ids,
            std::map<int64_t, int64_t> const *i_dim_sizes_inner,
            std::map<int64_t, int64_t> const *i_dim_sizes_aux_outer,
            std::map<int64_t, int64_t> const *i_dim_sizes_outer,
            std::map<int64_t, int64_t> const *i_offsets_aux,
            std::map<int64_t, int64_t> const *i_offsets, data_t i_dtype, void *i_data_ptr_aux,
            void *i_data_ptr, kernel_t i_ktype_first_touch, kernel_t i_ktype_main,
            kernel_t i_ktype_last_touch, EinsumNode *i_left, EinsumNode *i_right,
            MemoryManager *i_memory, int64_t i_num_threads);

  err_t compile();
  err_t compile_recursive();
  err_t store_and_lock_data();
  err_t unlock_data();
  //! enqueues the evaluation of the subtree; returns the first error status (extension)
  int eval();
  int64_t num_ops(bool i_children = true);
  void cancel_memory_reservation();
  void compile_memory_usage();
  bool requires_permutation();
  //! sets the stream of this node and its subtree (extension)
  void set_stream(void *i_stream);
};

}  // namespace backend
}  // namespace einsum_ir

#endif
