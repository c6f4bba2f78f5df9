// Device arena for the intermediate tensors of an einsum tree.
//
// Same two-ended stack discipline as the reference's backend::MemoryManager
// (src/backend/MemoryManager.cpp:9-106): tensors reserved while compiling an
// even tree layer grow from the left end, odd layers from the right end, so a
// node's output and its children's outputs never overlap while both are live.
// One allocation of the peak size is made by alloc_all_memory (device memory,
// cudaMalloc); get_mem_ptr turns a reservation id into a device pointer.
#ifndef EINSUM_IR_B200_MEMORY_MANAGER_H
#define EINSUM_IR_B200_MEMORY_MANAGER_H

#include <cstdint>
#include <list>
#include <vector>
#include "constants.h"

namespace einsum_ir {
namespace backend {

class MemoryManager {
 public:
  //! layer of the tree being compiled (even: left end, odd: right end)
  int64_t m_layer_id = 0;
  //! peak bytes needed by all reservations (excluding alignment slack)
  int64_t m_req_mem = 0;

  ~MemoryManager();

  //! reserves i_size bytes (rounded up to the line alignment); returns the id
  //! (positive: left end, negative: right end)
  int64_t reserve_memory(int64_t i_size);

  //! ends the reservation with the given id
  void remove_reservation(int64_t i_id);

  //! allocates the device arena of the peak size (once)
  err_t alloc_all_memory();

  //! device pointer of a reservation (valid after alloc_all_memory)
  void *get_mem_ptr(int64_t i_id);

  int64_t alignment_line() const { return m_alignment_line; }

 private:
  int64_t m_alignment_line = 256;
  int64_t m_alignment_page = 4096;
  char *m_memory_ptr = nullptr;
  char *m_aligned_memory_ptr = nullptr;
  int64_t m_allocated_bytes = 0;
  int64_t m_last_id = 0;
  std::vector<int64_t> m_tensor_offset;
  std::list<int64_t> m_allocated_id_left, m_allocated_id_right;
  std::list<int64_t> m_allocated_offset_left, m_allocated_offset_right;
};

}  // namespace backend
}  // namespace einsum_ir

#endif
