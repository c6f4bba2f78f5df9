// A binary contraction whose output's outermost dim is split into contiguous
// blocks over the GPUs of a node (one process per GPU): this backend's C++
// entry point for BASELINE config 5 (zabcd,zcdef->zabef, z sharded). The
// reference has no multi-GPU path; the interface follows its
// BinaryContraction (dim ids, sizes maps, init / compile / contract /
// num_ops), plus the sharded dim and the rank layout.
//
// Rank r computes block r of the sharded dim (size / world slabs) with one
// plan and eir_contract_gather: the copy engines push every finished slab of
// the block into the other ranks' full outputs (mapped once by
// bind_output through the caller's all-gather), while the kernel computes
// the next slabs. After the contract call has passed the stream on every rank
// (stream synchronisation, then a cross-rank barrier), every rank holds the
// full output.
#ifndef EINSUM_IR_B200_SHARDED_CONTRACTION_H
#define EINSUM_IR_B200_SHARDED_CONTRACTION_H

#include <map>
#include <vector>
#include "BinaryContractionCuda.h"
#include "MemoryManager.h"
#include "eir_cuda.h"

namespace einsum_ir {
namespace backend {

class ShardedContraction {
 public:
  ~ShardedContraction();

  //! the contraction as BinaryContraction::init would take it (sizes of all
  //! dims; tensors row-major in the order of their ids), the id of the
  //! sharded dim (outermost in the output and in every input holding it),
  //! and this process's rank among `world` ranks
  void init(int64_t i_num_dims_left, int64_t i_num_dims_right, int64_t i_num_dims_out,
            std::map<int64_t, int64_t> const *i_dim_sizes, int64_t const *i_dim_ids_left,
            int64_t const *i_dim_ids_right, int64_t const *i_dim_ids_out, data_t i_dtype,
            int64_t i_shard_dim_id, int32_t i_rank, int32_t i_world);
  void set_compute_type(int32_t i_comp) { m_comp = i_comp; }
  void set_stream(void *i_stream) { m_stream = i_stream; }

  //! the plan of this rank's block
  err_t compile();
  //! maps every rank's full output `io_out_full` (same size on every rank)
  //! into this process; collective over the ranks through `i_allgather`
  int bind_output(void *io_out_full, eir_allgather_fn i_allgather, void *i_user);
  //! this rank's block of the inputs (pointers to the block, or to the whole
  //! tensor if it does not hold the sharded dim) into io_out_full, gathered
  //! into every rank's full output; asynchronous on the stream
  int contract(void const *i_left_block, void const *i_right_block, void *io_out_full);
  //! closes the peer mappings (every rank, before any rank frees its output)
  void unbind();

  //! flops of the whole job (all ranks)
  int64_t num_ops() const;
  //! slabs of the sharded dim this rank computes: [block_begin, block_begin + block_size)
  int64_t block_begin() const { return m_block * m_rank; }
  int64_t block_size() const { return m_block; }
  //! bytes of one index of the sharded dim in the output
  int64_t slab_bytes() const { return m_slab_bytes; }

 private:
  std::vector<int64_t> m_ids_l, m_ids_r, m_ids_o;
  std::map<int64_t, int64_t> m_sizes_block;
  data_t m_dtype = UNDEFINED_DTYPE;
  int64_t m_shard = -1, m_block = 0, m_slab_bytes = 0;
  int32_t m_rank = 0, m_world = 1, m_comp = EIR_COMPUTE_DEFAULT;
  void *m_stream = nullptr;
  MemoryManager m_memory;
  BinaryContractionCuda m_block_contraction;
  eir_output_group *m_group = nullptr;
  void *m_bound = nullptr;
  bool m_compiled = false;
};

}  // namespace backend
}  // namespace einsum_ir

#endif
