#include "Unary.h"

namespace einsum_ir {
namespace backend {

void Unary::strides(int64_t i_num_dims, std::map<int64_t, int64_t> const *i_dim_sizes,
                    int64_t const *i_dim_ids, int64_t *o_strides) {
  int64_t s = 1;
  for (int64_t d = i_num_dims - 1; d >= 0; --d) {
    o_strides[d] = s;
    s *= i_dim_sizes->at(i_dim_ids[d]);
  }
}

void Unary::order_strides_output_based(int64_t i_num_dims, int64_t const *i_dim_ids_in,
                                       int64_t const *i_dim_ids_out, int64_t *io_strides) {
  std::map<int64_t, int64_t> by_id;
  for (int64_t d = 0; d < i_num_dims; ++d) by_id.insert({i_dim_ids_in[d], io_strides[d]});
  for (int64_t d = 0; d < i_num_dims; ++d) io_strides[d] = by_id.at(i_dim_ids_out[d]);
}

void Unary::init(int64_t i_num_dims, std::map<int64_t, int64_t> const *i_dim_sizes,
                 int64_t const *i_dim_ids_in, int64_t const *i_dim_ids_out, data_t i_dtype_in,
                 data_t i_dtype_comp, data_t i_dtype_out, kernel_t i_ktype_main,
                 int64_t i_num_threads) {
  m_num_dims = i_num_dims;
  m_dim_sizes = i_dim_sizes;
  m_dim_ids_in = i_dim_ids_in;
  m_dim_ids_out = i_dim_ids_out;
  m_dtype_in = i_dtype_in;
  m_dtype_comp = i_dtype_comp;
  m_dtype_out = i_dtype_out;
  m_ktype_main = i_ktype_main;
  m_num_threads = i_num_threads;
}

UnaryCuda::~UnaryCuda() {
  if (m_plan != nullptr) eir_plan_destroy(m_plan);
}

err_t UnaryCuda::compile() {
  if (m_ktype_main != COPY) return INVALID_KTYPE;
  if (m_dtype_in != m_dtype_out) return INVALID_DTYPE;
  m_strides_in.assign(m_num_dims, 0);
  m_strides_out.assign(m_num_dims, 0);
  std::vector<int64_t> sizes(m_num_dims);
  if (m_num_dims > 0) {
    strides(m_num_dims, m_dim_sizes, m_dim_ids_in, m_strides_in.data());
    order_strides_output_based(m_num_dims, m_dim_ids_in, m_dim_ids_out, m_strides_in.data());
    strides(m_num_dims, m_dim_sizes, m_dim_ids_out, m_strides_out.data());
    for (int64_t d = 0; d < m_num_dims; ++d) sizes[d] = m_dim_sizes->at(m_dim_ids_out[d]);
  }
  if (m_plan != nullptr) eir_plan_destroy(m_plan);
  m_plan = nullptr;
  int rc = eir_permute_plan_create((int32_t)m_num_dims, sizes.data(), m_strides_in.data(),
                                   m_strides_out.data(), (int32_t)m_dtype_in, &m_plan);
  if (rc != EIR_SUCCESS) return rc == EIR_INVALID_DTYPE ? INVALID_DTYPE : COMPILATION_FAILED;
  m_compiled = true;
  return SUCCESS;
}

void UnaryCuda::eval(void const *i_tensor_in, void *io_tensor_out) {
  if (!m_compiled) {
    m_last_status = EIR_CALLED_BEFORE_COMPILATION;
    return;
  }
  m_last_status = eir_permute(m_plan, i_tensor_in, io_tensor_out, m_stream);
}

}  // namespace backend
}  // namespace einsum_ir
