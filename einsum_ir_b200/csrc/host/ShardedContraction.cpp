#include "ShardedContraction.h"

#include <vector>

namespace einsum_ir {
namespace backend {

ShardedContraction::~ShardedContraction() { unbind(); }

void ShardedContraction::init(int64_t i_num_dims_left, int64_t i_num_dims_right, int64_t i_num_dims_out,
                              std::map<int64_t, int64_t> const *i_dim_sizes, int64_t const *i_dim_ids_left,
                              int64_t const *i_dim_ids_right, int64_t const *i_dim_ids_out, data_t i_dtype,
                              int64_t i_shard_dim_id, int32_t i_rank, int32_t i_world) {
  m_ids_l.assign(i_dim_ids_left, i_dim_ids_left + i_num_dims_left);
  m_ids_r.assign(i_dim_ids_right, i_dim_ids_right + i_num_dims_right);
  m_ids_o.assign(i_dim_ids_out, i_dim_ids_out + i_num_dims_out);
  m_sizes_block = *i_dim_sizes;
  m_dtype = i_dtype;
  m_shard = i_shard_dim_id;
  m_rank = i_rank;
  m_world = i_world;
  m_compiled = false;
}

err_t ShardedContraction::compile() {
  if (m_world < 1 || m_rank < 0 || m_rank >= m_world || m_ids_o.empty() || m_ids_o[0] != m_shard)
    return COMPILATION_FAILED;
  for (auto const *ids : {&m_ids_l, &m_ids_r})
    for (size_t d = 0; d < ids->size(); ++d)
      if ((*ids)[d] == m_shard && d != 0) return DIMENSION_ORDERING_FAILED;  // must be outermost
  auto it = m_sizes_block.find(m_shard);
  if (it == m_sizes_block.end() || it->second % m_world != 0) return COMPILATION_FAILED;
  m_block = it->second / m_world;
  it->second = m_block;
  int64_t slab = m_dtype == FP64 ? 8 : 4;
  for (size_t d = 1; d < m_ids_o.size(); ++d) slab *= m_sizes_block.at(m_ids_o[d]);
  m_slab_bytes = slab;
  m_block_contraction.init((int64_t)m_ids_l.size(), (int64_t)m_ids_r.size(), (int64_t)m_ids_o.size(),
                           &m_sizes_block, &m_sizes_block, &m_sizes_block, nullptr, &m_sizes_block, nullptr,
                           m_ids_l.data(), m_ids_r.data(), m_ids_o.data(), nullptr, nullptr, &m_memory, m_dtype,
                           m_dtype, m_dtype, m_dtype, ZERO, MADD, UNDEFINED_KTYPE, 1);
  m_block_contraction.set_compute_type(m_comp);
  m_block_contraction.set_stream(m_stream);
  err_t err = m_block_contraction.compile();
  m_compiled = err == SUCCESS;
  return err;
}

int ShardedContraction::bind_output(void *io_out_full, eir_allgather_fn i_allgather, void *i_user) {
  unbind();
  int rc = eir_output_group_create(m_rank, m_world, io_out_full, i_allgather, i_user, &m_group);
  if (rc == EIR_SUCCESS) m_bound = io_out_full;
  return rc;
}

void ShardedContraction::unbind() {
  if (m_group != nullptr) eir_output_group_destroy(m_group);
  m_group = nullptr;
  m_bound = nullptr;
}

int ShardedContraction::contract(void const *i_left_block, void const *i_right_block, void *io_out_full) {
  if (!m_compiled) return CALLED_BEFORE_COMPILATION;
  if (io_out_full == nullptr || io_out_full != m_bound) return EIR_INVALID_ARGUMENT;  // bind_output first
  const int64_t offset = block_begin() * m_slab_bytes;
  std::vector<void *> peers((size_t)(m_world > 1 ? m_world - 1 : 1), nullptr);
  int rc = eir_output_group_peers(m_group, offset, peers.data());
  if (rc != EIR_SUCCESS) return rc;
  return eir_contract_gather(m_block_contraction.m_plan, i_left_block, i_right_block, nullptr,
                             static_cast<char *>(io_out_full) + offset, m_world - 1, peers.data(), m_stream);
}

int64_t ShardedContraction::num_ops() const {
  return m_compiled ? eir_contract_num_ops(m_block_contraction.m_plan) * m_world : 0;
}

}  // namespace backend
}  // namespace einsum_ir
