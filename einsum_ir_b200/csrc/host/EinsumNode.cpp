// Tree compile / memory plan / eval, following the control flow of the
// reference's src/backend/EinsumNode.cpp (line ranges per function), with the
// CUDA backend for contractions and permutes and a device arena.
#include "EinsumNode.h"

#include <cuda_runtime.h>
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include "BinaryContractionCuda.h"
#include "BinaryPrimitives.h"

namespace einsum_ir {
namespace backend {

namespace {
bool env_flag(char const *name, bool dflt) {
  char const *v = std::getenv(name);
  if (v == nullptr) return dflt;
  return std::strcmp(v, "1") == 0 || std::strcmp(v, "true") == 0;
}
}  // namespace

EinsumNode::~EinsumNode() {
  delete m_unary;
  delete m_cont;
  if (m_data_ptr_int != nullptr) cudaFree(m_data_ptr_int);
}

// input node (reference :21-125): backend and layout flags from the environment
void EinsumNode::init(int64_t i_num_dims, int64_t const *i_dim_ids,
                      std::map<int64_t, int64_t> const *i_dim_sizes_inner,
                      std::map<int64_t, int64_t> const *i_dim_sizes_outer, data_t i_dtype,
                      void *i_data_ptr, MemoryManager *i_memory) {
  m_dtype = i_dtype;
  m_ktype_first_touch = m_ktype_main = m_ktype_last_touch = UNDEFINED_KTYPE;
  m_size = 0;
  m_num_dims = i_num_dims;
  m_dim_ids_ext = i_dim_ids;
  m_dim_ids_int.assign(i_dim_ids, i_dim_ids + i_num_dims);
  m_dim_sizes_inner = i_dim_sizes_inner;
  m_dim_sizes_outer = i_dim_sizes_outer != nullptr ? i_dim_sizes_outer : i_dim_sizes_inner;
  m_offsets_aux_ext = m_offsets_ext = nullptr;
  m_children.clear();
  m_data_ptr_int = m_data_ptr_active = nullptr;
  m_data_ptr_ext = i_data_ptr;

  m_btype_unary = AUTO;
  m_btype_binary = AUTO;
  if (char const *b = std::getenv("EINSUM_IR_BACKEND")) {
    if (!std::strcmp(b, "AUTO")) m_btype_binary = AUTO;
    else if (!std::strcmp(b, "CUDA")) m_btype_binary = CUDA;
    else if (!std::strcmp(b, "TPP")) m_btype_binary = TPP;
    else if (!std::strcmp(b, "BLAS")) m_btype_binary = BLAS;
    else if (!std::strcmp(b, "TBLIS")) m_btype_binary = TBLIS;
    else if (!std::strcmp(b, "SCALAR")) m_btype_binary = SCALAR;
  }
  m_reorder_dims = env_flag("EINSUM_IR_REORDER_DIMS", true);
  m_pack_inputs = env_flag("EINSUM_IR_PACK_INPUTS", false);
  m_unary = nullptr;
  m_cont = nullptr;
  m_num_ops_node = m_num_ops_children = 0;
  m_num_tasks_intra_op = 1;
  m_memory = i_memory;
  m_mem_id = 0;
  m_count_mem_users = 1;
  m_active_mem_users = 0;
  m_req_mem = m_mem_subtree = 0;
  m_compiled = m_data_locked = false;
}

void EinsumNode::init(int64_t i_num_dims, int64_t const *i_dim_ids,
                      std::map<int64_t, int64_t> const *i_dim_sizes_inner,
                      std::map<int64_t, int64_t> const *i_dim_sizes_outer, data_t i_dtype,
                      void *i_data_ptr, EinsumNode *i_child, MemoryManager *i_memory,
                      int64_t i_num_threads) {
  init(i_num_dims, i_dim_ids, i_dim_sizes_inner, i_dim_sizes_outer, i_dtype, i_data_ptr, i_memory);
  m_children = {i_child};
  m_num_threads = i_num_threads;
}

void EinsumNode::init(int64_t i_num_dims, int64_t const *i_dim_ids,
                      std::map<int64_t, int64_t> const *i_dim_sizes_inner,
                      std::map<int64_t, int64_t> const *i_dim_sizes_aux_outer,
                      std::map<int64_t, int64_t> const *i_dim_sizes_outer,
                      std::map<int64_t, int64_t> const *i_offsets_aux,
                      std::map<int64_t, int64_t> const *i_offsets, data_t i_dtype,
                      void *i_data_ptr_aux, void *i_data_ptr, kernel_t i_ktype_first_touch,
                      kernel_t i_ktype_main, kernel_t i_ktype_last_touch, EinsumNode *i_left,
                      EinsumNode *i_right, MemoryManager *i_memory, int64_t i_num_threads) {
  init(i_num_dims, i_dim_ids, i_dim_sizes_inner, i_dim_sizes_outer, i_dtype, i_data_ptr, i_memory);
  m_dim_sizes_aux_outer = i_dim_sizes_aux_outer;
  m_offsets_aux_ext = i_offsets_aux;
  m_offsets_ext = i_offsets;
  m_data_ptr_aux_ext = i_data_ptr_aux;
  m_ktype_first_touch = i_ktype_first_touch;
  m_ktype_main = i_ktype_main;
  m_ktype_last_touch = i_ktype_last_touch;
  m_children = {i_left, i_right};
  m_num_threads = i_num_threads;
}

err_t EinsumNode::compile() {
  err_t err = compile_recursive();
  if (err != SUCCESS) return err;
  compile_memory_usage();
  return m_memory->alloc_all_memory();
}

// reference :204-454
err_t EinsumNode::compile_recursive() {
  if (m_btype_binary == AUTO) m_btype_binary = CUDA;
  if (m_btype_binary != CUDA) return INVALID_BACKEND;
  // complex contractions: CPX_ZERO / CPX_MADD (validated by the contraction)
  const bool cpx_pair = m_ktype_main == CPX_MADD &&
                        (m_ktype_first_touch == CPX_ZERO || m_ktype_first_touch == UNDEFINED_KTYPE) &&
                        m_ktype_last_touch == UNDEFINED_KTYPE;
  if (!cpx_pair &&
      (ce_cpx_op(m_ktype_first_touch) || ce_cpx_op(m_ktype_main) || ce_cpx_op(m_ktype_last_touch)))
    return INVALID_KTYPE;

  m_size = ce_n_bytes(m_dtype);
  for (int64_t d = 0; d < m_num_dims; ++d) m_size *= m_dim_sizes_outer->at(m_dim_ids_ext[d]);

  if (m_children.size() == 2) {
    if (BinaryPrimitives::swap_inputs(m_children[0]->m_num_dims, m_children[1]->m_num_dims,
                                      m_num_dims, m_children[0]->m_dim_ids_ext,
                                      m_children[1]->m_dim_ids_ext, m_dim_ids_int.data()))
      std::swap(m_children[0], m_children[1]);
    if (m_reorder_dims) {
      // only intermediate results are laid out freely (no permute cost)
      bool left_free = !m_children[0]->m_children.empty();
      bool right_free = !m_children[1]->m_children.empty();
      err_t err = BinaryPrimitives::reorder(
          m_children[0]->m_num_dims, m_children[1]->m_num_dims, m_num_dims, m_dim_sizes_inner,
          left_free, right_free, m_children[0]->m_dim_ids_int.data(),
          m_children[1]->m_dim_ids_int.data(), m_dim_ids_int.data());
      if (err != SUCCESS) return err;
    }
    auto *cont = new BinaryContractionCuda();
    cont->set_compute_type(m_compute);
    cont->set_stream(m_stream);
    m_cont = cont;
    m_cont->init(m_children[0]->m_num_dims, m_children[1]->m_num_dims, m_num_dims,
                 m_dim_sizes_inner, m_children[0]->m_dim_sizes_outer,
                 m_children[1]->m_dim_sizes_outer, m_dim_sizes_aux_outer, m_dim_sizes_outer, nullptr,
                 m_children[0]->m_dim_ids_int.data(), m_children[1]->m_dim_ids_int.data(),
                 m_dim_ids_int.data(), nullptr, nullptr, m_memory, m_children[0]->m_dtype,
                 m_children[1]->m_dtype, m_dtype, m_dtype, m_ktype_first_touch, m_ktype_main,
                 m_ktype_last_touch, m_num_threads);
    err_t err = m_cont->compile();
    if (err != SUCCESS) return err;
  }

  // permute: external -> internal order (input nodes), child -> this (unary nodes)
  auto *unary = new UnaryCuda();
  unary->set_stream(m_stream);
  m_unary = unary;
  if (m_children.size() != 1)
    m_unary->init(m_num_dims, m_dim_sizes_outer, m_dim_ids_ext, m_dim_ids_int.data(), m_dtype,
                  m_dtype, m_dtype, COPY, 1);
  else
    m_unary->init(m_num_dims, m_dim_sizes_outer, m_children[0]->m_dim_ids_ext, m_dim_ids_ext,
                  m_dtype, m_dtype, m_dtype, COPY, 1);
  err_t err = m_unary->compile();
  if (err != SUCCESS) return err;

  // byte offsets into the data / aux tensors (reference :359-391; the aux offset
  // is accumulated into the aux offset here)
  auto offset = [&](std::map<int64_t, int64_t> const *offs, std::map<int64_t, int64_t> const *outer) {
    int64_t o = 0, s = 1;
    for (int64_t d = m_num_dims - 1; d >= 0; --d) {
      int64_t id = m_dim_ids_int[d];
      auto it = offs->find(id);
      if (it != offs->end()) o += s * it->second;
      s *= outer->at(id);
    }
    return o * ce_n_bytes(m_dtype);
  };
  if (m_offsets_aux_ext != nullptr && m_dim_sizes_aux_outer != nullptr)
    m_offset_aux_bytes = offset(m_offsets_aux_ext, m_dim_sizes_aux_outer);
  if (m_offsets_ext != nullptr) m_offset_bytes = offset(m_offsets_ext, m_dim_sizes_outer);

  m_req_mem = (m_data_ptr_ext == nullptr || requires_permutation()) ? m_size : 0;

  // children first, then the execution order with the lower peak memory (reference :393-437)
  if (m_children.size() == 2) {
    for (auto *ch : m_children) {
      err = ch->compile_recursive();
      if (err != SUCCESS) return err;
    }
    int64_t m0 = m_children[0]->m_mem_subtree, m1 = m_children[1]->m_mem_subtree;
    int64_t peak01 = std::max(m0, m1 + m_children[0]->m_req_mem);
    int64_t peak10 = std::max(m1, m0 + m_children[1]->m_req_mem);
    if (peak01 <= peak10) {
      m_mem_subtree = peak01;
      m_exec_order = {0, 1};
    } else {
      m_mem_subtree = peak10;
      m_exec_order = {1, 0};
    }
    m_mem_subtree = std::max(m_mem_subtree,
                             m_req_mem + m_children[0]->m_req_mem + m_children[1]->m_req_mem);
  } else if (m_children.size() == 1) {
    err = m_children[0]->compile_recursive();
    if (err != SUCCESS) return err;
    m_exec_order = {0};
    m_mem_subtree = std::max(m_children[0]->m_mem_subtree, m_req_mem + m_children[0]->m_req_mem);
  } else {
    m_mem_subtree = m_req_mem;
  }

  m_num_ops_node = m_children.size() == 2 ? m_cont->num_ops() : 0;
  m_num_ops_children = 0;
  for (auto *ch : m_children) m_num_ops_children += ch->m_num_ops_node + ch->m_num_ops_children;
  m_compiled = true;
  return SUCCESS;
}

// reference :458-479: a one-time permute of the input into node-owned device memory
err_t EinsumNode::store_and_lock_data() {
  if (!m_compiled) return CALLED_BEFORE_COMPILATION;
  if (m_data_ptr_ext == nullptr) return NO_DATA_PTR_PROVIDED;
  if (m_data_ptr_int == nullptr && cudaMalloc(&m_data_ptr_int, (size_t)std::max<int64_t>(m_size, 1)) != cudaSuccess) {
    m_data_ptr_int = nullptr;
    return COMPILATION_FAILED;
  }
  m_unary->eval(m_data_ptr_ext, m_data_ptr_int);
  if (static_cast<UnaryCuda *>(m_unary)->m_last_status != EIR_SUCCESS) return UNDEFINED_ERROR;
  m_data_locked = true;
  return SUCCESS;
}

err_t EinsumNode::unlock_data() {
  if (m_data_ptr_ext == nullptr) return NO_DATA_PTR_PROVIDED;
  if (m_data_ptr_int != nullptr) {
    cudaStreamSynchronize(static_cast<cudaStream_t>(m_stream));
    cudaFree(m_data_ptr_int);
    m_data_ptr_int = nullptr;
  }
  m_data_locked = false;
  return SUCCESS;
}

// reference :496-540
int EinsumNode::eval() {
  int status = EIR_SUCCESS;
  for (size_t c = 0; c < m_children.size(); ++c) {
    int s = m_children[m_exec_order[c]]->eval();
    if (status == EIR_SUCCESS) status = s;
  }
  if (m_data_locked) {
    m_data_ptr_active = m_data_ptr_int;
  } else if (m_mem_id) {
    m_data_ptr_active = m_memory->get_mem_ptr(m_mem_id);
    m_active_mem_users = m_count_mem_users;
  } else {
    m_data_ptr_active = m_data_ptr_ext;
  }
  auto *unary = static_cast<UnaryCuda *>(m_unary);
  if (m_children.size() != 1) {
    if (!m_data_locked && m_data_ptr_ext != nullptr && m_req_mem != 0) {
      unary->eval(m_data_ptr_ext, m_data_ptr_active);
      if (status == EIR_SUCCESS) status = unary->m_last_status;
    }
  } else {
    unary->eval(m_children[0]->m_data_ptr_active, m_data_ptr_active);
    if (status == EIR_SUCCESS) status = unary->m_last_status;
  }
  if (m_children.size() == 2) {
    void const *aux = m_data_ptr_aux_int != nullptr ? m_data_ptr_aux_int : m_data_ptr_aux_ext;
    if (aux != nullptr) aux = static_cast<char const *>(aux) + m_offset_aux_bytes;
    void *out = static_cast<char *>(m_data_ptr_active) + m_offset_bytes;
    m_cont->contract(m_children[0]->m_data_ptr_active, m_children[1]->m_data_ptr_active, aux, out);
    if (status == EIR_SUCCESS) status = static_cast<BinaryContractionCuda *>(m_cont)->m_last_status;
  }
  return status;
}

int64_t EinsumNode::num_ops(bool i_children) {
  return m_num_ops_node + (i_children ? m_num_ops_children : 0);
}

void EinsumNode::cancel_memory_reservation() {
  m_active_mem_users--;
  if (m_active_mem_users <= 0 && m_mem_id) m_memory->remove_reservation(m_mem_id);
}

// reference :552-578: children reserve in layer+1, the node in its own layer
void EinsumNode::compile_memory_usage() {
  m_memory->m_layer_id++;
  for (size_t c = 0; c < m_children.size(); ++c) m_children[m_exec_order[c]]->compile_memory_usage();
  m_memory->m_layer_id--;
  if (m_req_mem) m_mem_id = m_memory->reserve_memory(m_req_mem);
  for (auto *ch : m_children) ch->cancel_memory_reservation();
}

bool EinsumNode::requires_permutation() {
  if (m_dim_ids_ext == m_dim_ids_int.data() || m_data_ptr_ext == nullptr) return false;
  for (int64_t d = 0; d < m_num_dims; ++d)
    if (m_dim_ids_ext[d] != m_dim_ids_int[d]) return true;
  return false;
}

void EinsumNode::set_stream(void *i_stream) {
  m_stream = i_stream;
  if (m_cont) static_cast<BinaryContractionCuda *>(m_cont)->set_stream(i_stream);
  if (m_unary) static_cast<UnaryCuda *>(m_unary)->set_stream(i_stream);
  for (auto *ch : m_children) ch->set_stream(i_stream);
}

}  // namespace backend
}  // namespace einsum_ir
