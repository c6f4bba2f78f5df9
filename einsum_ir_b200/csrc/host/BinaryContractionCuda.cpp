#include "BinaryContractionCuda.h"

#include <vector>

namespace einsum_ir {
namespace backend {

BinaryContractionCuda::~BinaryContractionCuda() {
  if (m_plan != nullptr) eir_plan_destroy(m_plan);
}

err_t BinaryContractionCuda::compile() {
  err_t err = compile_base();
  if (err != SUCCESS) return err;
  if (m_num_dims_i > 0 || m_num_dims_j > 0) return COMPILATION_FAILED;  // no one-sided sums
  // complex contractions: CPX_ZERO (or accumulate) + CPX_MADD, no last touch.
  // The complex dim is the size-2 C dim with the largest id (the frontends add
  // it after the real dims, src/bench_expression.cpp:110).
  const bool cpx = m_ktype_main == CPX_MADD;
  if (cpx ? ((m_ktype_first_touch != CPX_ZERO && m_ktype_first_touch != UNDEFINED_KTYPE) ||
             m_ktype_last_touch != UNDEFINED_KTYPE)
          : (ce_cpx_op(m_ktype_first_touch) || ce_cpx_op(m_ktype_main) || ce_cpx_op(m_ktype_last_touch)))
    return INVALID_KTYPE;
  int64_t cpx_id = -1;
  if (cpx) {
    for (size_t d = 0; d < m_dim_ids_c.size(); ++d)
      if (m_sizes_c[d] == 2 && m_dim_ids_c[d] > cpx_id) cpx_id = m_dim_ids_c[d];
    if (cpx_id < 0) return INVALID_CPX_DIM;
  }

  // strides as in the reference backends (BinaryContractionTpp.cpp:12-42): row-major
  // from the outer sizes; the aux tensor uses its own outer sizes, or the output's
  // when a touch kernel reads it and none were given
  std::map<int64_t, int64_t> sl, sr, so, sa;
  strides(m_num_dims_left, m_dim_ids_left, m_dim_sizes_outer_left, &sl);
  strides(m_num_dims_right, m_dim_ids_right, m_dim_sizes_outer_right, &sr);
  strides(m_num_dims_out, m_dim_ids_out, m_dim_sizes_outer_out, &so);
  if (m_dim_sizes_outer_out_aux != nullptr)
    strides(m_num_dims_out, m_dim_ids_out, m_dim_sizes_outer_out_aux, &sa);
  else if (m_ktype_first_touch == ADD || m_ktype_first_touch == COPY || m_ktype_last_touch == ADD)
    sa = so;
  auto get = [](std::map<int64_t, int64_t> const &m, int64_t id) {
    auto it = m.find(id);
    return it == m.end() ? int64_t(0) : it->second;
  };

  std::vector<eir_dim> dims;
  auto add = [&](std::vector<int64_t> const &ids, std::vector<int64_t> const &sizes, int32_t type) {
    for (size_t d = 0; d < ids.size(); ++d) {
      eir_dim x{};
      x.type = ids[d] == cpx_id ? EIR_DIM_CPX : type;
      x.size = sizes[d];
      x.stride_left = get(sl, ids[d]);
      x.stride_right = get(sr, ids[d]);
      x.stride_out = get(so, ids[d]);
      x.stride_out_aux = get(sa, ids[d]);
      dims.push_back(x);
    }
  };
  add(m_dim_ids_c, m_sizes_c, EIR_DIM_C);
  add(m_dim_ids_m, m_sizes_m, EIR_DIM_M);
  add(m_dim_ids_n, m_sizes_n, EIR_DIM_N);
  add(m_dim_ids_k, m_sizes_k, EIR_DIM_K);

  eir_contract_desc desc{};
  desc.num_dims = (int32_t)dims.size();
  desc.dims = dims.data();
  desc.dtype_left = (int32_t)m_dtype_left;
  desc.dtype_right = (int32_t)m_dtype_right;
  desc.dtype_out = (int32_t)m_dtype_out;
  desc.dtype_comp = m_comp;
  desc.ktype_first_touch = (int32_t)m_ktype_first_touch;
  desc.ktype_main = (int32_t)(m_ktype_main == UNDEFINED_KTYPE ? MADD : m_ktype_main);
  desc.ktype_last_touch = (int32_t)m_ktype_last_touch;
  desc.flags = m_flags;
  if (m_plan != nullptr) {
    eir_plan_destroy(m_plan);
    m_plan = nullptr;
  }
  int rc = eir_contract_plan_create(&desc, &m_plan);
  if (rc != EIR_SUCCESS) return rc == EIR_INVALID_DTYPE ? INVALID_DTYPE
                                : rc == EIR_INVALID_KTYPE ? INVALID_KTYPE
                                : rc == EIR_INVALID_CPX_DIM ? INVALID_CPX_DIM
                                                          : COMPILATION_FAILED;
  m_compiled = true;
  return SUCCESS;
}

void BinaryContractionCuda::contract(void const *i_tensor_left, void const *i_tensor_right,
                                     void *io_tensor_out) {
  contract(i_tensor_left, i_tensor_right, nullptr, io_tensor_out);
}

void BinaryContractionCuda::contract(void const *i_tensor_left, void const *i_tensor_right,
                                     void const *i_tensor_out_aux, void *io_tensor_out) {
  if (!m_compiled || m_plan == nullptr) {
    m_last_status = EIR_CALLED_BEFORE_COMPILATION;
    return;
  }
  m_last_status = eir_contract(m_plan, i_tensor_left, i_tensor_right, i_tensor_out_aux,
                               io_tensor_out, m_stream);
}

}  // namespace backend
}  // namespace einsum_ir
