#include "MemoryManager.h"

#include <cuda_runtime.h>

namespace einsum_ir {
namespace backend {

MemoryManager::~MemoryManager() {
  if (m_memory_ptr != nullptr) cudaFree(m_memory_ptr);
}

int64_t MemoryManager::reserve_memory(int64_t i_size) {
  m_last_id++;
  if (i_size % m_alignment_line) i_size += m_alignment_line - i_size % m_alignment_line;
  int64_t id;
  if (m_layer_id % 2 == 0) {
    // left end grows upwards from offset 0
    int64_t top = m_allocated_offset_left.empty() ? 0 : m_allocated_offset_left.front();
    m_tensor_offset.push_back(top);
    id = m_last_id;
    m_allocated_id_left.push_front(id);
    m_allocated_offset_left.push_front(top + i_size);
  } else {
    // right end grows downwards from the end of the arena (negative offsets)
    int64_t bottom = m_allocated_offset_right.empty() ? 0 : m_allocated_offset_right.front();
    m_tensor_offset.push_back(bottom - i_size);
    id = -m_last_id;
    m_allocated_id_right.push_front(id);
    m_allocated_offset_right.push_front(bottom - i_size);
  }
  int64_t left = m_allocated_offset_left.empty() ? 0 : m_allocated_offset_left.front();
  int64_t right = m_allocated_offset_right.empty() ? 0 : m_allocated_offset_right.front();
  if (left - right > m_req_mem) m_req_mem = left - right;
  return id;
}

void MemoryManager::remove_reservation(int64_t i_id) {
  auto &ids = i_id >= 0 ? m_allocated_id_left : m_allocated_id_right;
  auto &offs = i_id >= 0 ? m_allocated_offset_left : m_allocated_offset_right;
  auto it_id = ids.begin();
  auto it_off = offs.begin();
  for (; it_id != ids.end(); ++it_id, ++it_off) {
    if (*it_id == i_id) {
      ids.erase(it_id);
      offs.erase(it_off);
      return;
    }
  }
}

err_t MemoryManager::alloc_all_memory() {
  if (m_req_mem == 0 || m_allocated_bytes >= m_req_mem) return SUCCESS;
  if (m_memory_ptr != nullptr) cudaFree(m_memory_ptr);
  m_memory_ptr = nullptr;
  size_t bytes = (size_t)(m_req_mem + m_alignment_page);
  if (cudaMalloc(reinterpret_cast<void **>(&m_memory_ptr), bytes) != cudaSuccess) {
    m_memory_ptr = nullptr;
    return COMPILATION_FAILED;
  }
  uintptr_t p = reinterpret_cast<uintptr_t>(m_memory_ptr);
  uintptr_t pad = (m_alignment_page - p % m_alignment_page) % m_alignment_page;
  m_aligned_memory_ptr = m_memory_ptr + pad;
  m_allocated_bytes = m_req_mem;
  return SUCCESS;
}

void *MemoryManager::get_mem_ptr(int64_t i_id) {
  if (m_aligned_memory_ptr == nullptr || i_id == 0) return nullptr;
  if (i_id > 0) return m_aligned_memory_ptr + m_tensor_offset[i_id - 1];
  return m_aligned_memory_ptr + m_req_mem + m_tensor_offset[-i_id - 1];
}

}  // namespace backend
}  // namespace einsum_ir
