// TensorOperation (reference: python/src/TensorOperation.cpp:1-771) on the
// B200 backend's C-ABI plans.
#include "TensorOperation.h"

#include <algorithm>
#include <cstdlib>
#include "eir_cuda.h"

namespace einsum_ir {
namespace py {

namespace {

using TO = TensorOperation;

// reference: determine_op_type, TensorOperation.cpp:5-18
TO::op_type_t op_type_of(TO::prim_t prim_main) {
  switch (prim_main) {
    case TO::prim_t::zero:
    case TO::prim_t::copy:
      return TO::op_type_t::unary;
    case TO::prim_t::gemm:
    case TO::prim_t::brgemm:
      return TO::op_type_t::binary;
    default:
      return TO::op_type_t::undefined;
  }
}

int32_t eir_dim_type(TO::dim_t d) {
  switch (d) {
    case TO::dim_t::c: return EIR_DIM_C;
    case TO::dim_t::m: return EIR_DIM_M;
    case TO::dim_t::n: return EIR_DIM_N;
    case TO::dim_t::k: return EIR_DIM_K;
    default: return -1;
  }
}

int32_t eir_dtype(TO::dtype_t d) {
  switch (d) {
    case TO::dtype_t::fp32: return EIR_FP32;
    case TO::dtype_t::fp64: return EIR_FP64;
  }
  return EIR_UNDEFINED_DTYPE;
}

// Shape checks shared by setup and optimize, in the reference's order
// (TensorOperation.cpp:229-262, 520-552): level 0 must exist, hold one
// stride vector per tensor, and each vector one stride per dimension.
TO::error_t check_level0(TO::op_type_t op, std::vector<int64_t> const &dim_sizes, TO::strides_t const &strides) {
  if (op == TO::op_type_t::undefined) return TO::error_t::compilation_failed;
  if (strides.empty()) return TO::error_t::invalid_stride_shape;
  const size_t tensors = op == TO::op_type_t::binary ? 3 : 2;
  if (strides[0].size() != tensors) return TO::error_t::invalid_stride_shape;
  for (auto const &t : strides[0])
    if (t.size() != dim_sizes.size()) return TO::error_t::invalid_stride_shape;
  return TO::error_t::success;
}

struct LoopDim {
  TO::dim_t type;
  int64_t size;
  int64_t s[3];  // in0, in1 (0 for unary), out
};

// drop size-1 dims and fuse (outer i, inner j) pairs of one type whose
// strides satisfy s_i = s_j * size_j in every tensor
std::vector<LoopDim> simplify(std::vector<LoopDim> d, int tensors) {
  std::vector<LoopDim> kept;
  for (auto const &x : d)
    if (x.size != 1) kept.push_back(x);
  if (kept.empty() && !d.empty()) kept.push_back(d.front());
  bool changed = true;
  while (changed) {
    changed = false;
    for (size_t i = 0; i < kept.size() && !changed; ++i)
      for (size_t j = 0; j < kept.size() && !changed; ++j) {
        if (i == j || kept[i].type != kept[j].type) continue;
        bool ok = true;
        for (int t = 0; t < tensors; ++t) ok = ok && kept[i].s[t] == kept[j].s[t] * kept[j].size;
        if (!ok) continue;
        kept[i].size *= kept[j].size;
        for (int t = 0; t < tensors; ++t) kept[i].s[t] = kept[j].s[t];
        kept.erase(kept.begin() + (long)j);
        changed = true;
      }
  }
  return kept;
}

// index of the dim of `type` with the smallest non-zero |stride| in tensor t, or -1
int innermost(std::vector<LoopDim> const &d, TO::dim_t type, int t) {
  int best = -1;
  for (size_t i = 0; i < d.size(); ++i) {
    if (d[i].type != type || d[i].s[t] == 0) continue;
    if (best < 0 || std::llabs(d[i].s[t]) < std::llabs(d[best].s[t])) best = (int)i;
  }
  return best;
}

}  // namespace

TO::op_type_t TensorOperation::determine_op_type(prim_t prim_main) { return op_type_of(prim_main); }

TensorOperation::~TensorOperation() { release(); }

void TensorOperation::release() {
  if (m_plan != nullptr) eir_plan_destroy(m_plan);
  m_plan = nullptr;
  m_op_type = op_type_t::undefined;
}

TO::error_t TensorOperation::setup(dtype_t dtype, prim_t prim_first, prim_t prim_main, prim_t prim_last,
                                   std::vector<dim_t> const &dim_types, std::vector<exec_t> const &exec_types,
                                   std::vector<int64_t> const &dim_sizes, strides_t const &strides) {
  release();
  const op_type_t op = op_type_of(prim_main);
  const error_t shape = check_level0(op, dim_sizes, strides);
  if (shape != error_t::success) return shape;
  // the reference leaves these mismatches undefined; here they fail to compile
  if (dim_types.size() != dim_sizes.size() || exec_types.size() != dim_sizes.size())
    return error_t::compilation_failed;
  for (auto e : exec_types)
    if (e == exec_t::undefined) return error_t::compilation_failed;
  const int32_t dt = eir_dtype(dtype);
  if (dt == EIR_UNDEFINED_DTYPE) return error_t::compilation_failed;
  const int32_t nd = (int32_t)dim_sizes.size();

  eir_plan *plan = nullptr;
  if (op == op_type_t::unary) {
    // reference: TensorOperation.cpp:276-281 (first / last touch must be none)
    if (prim_first != prim_t::none || prim_last != prim_t::none) return error_t::compilation_failed;
    const int32_t ktype = prim_main == prim_t::copy ? EIR_KTYPE_COPY : EIR_KTYPE_ZERO;
    if (eir_unary_plan_create(nd, dim_sizes.data(), strides[0][0].data(), strides[0][1].data(), dt, ktype,
                              &plan) != EIR_SUCCESS)
      return error_t::compilation_failed;
  } else {
    // reference: TensorOperation.cpp:334-457 (convert_prim_to_kernel: zero ->
    // ZERO, relu -> RELU, gemm / brgemm -> MADD / BR_MADD; none -> undefined)
    int32_t first = EIR_KTYPE_UNDEFINED, last = EIR_KTYPE_UNDEFINED;
    if (prim_first == prim_t::zero) first = EIR_KTYPE_ZERO;
    else if (prim_first != prim_t::none) return error_t::compilation_failed;
    if (prim_last == prim_t::relu) last = EIR_KTYPE_RELU;
    else if (prim_last != prim_t::none) return error_t::compilation_failed;
    std::vector<eir_dim> dims((size_t)nd);
    for (int32_t i = 0; i < nd; ++i) {
      const int32_t t = eir_dim_type(dim_types[(size_t)i]);
      if (t < 0) return error_t::compilation_failed;
      dims[(size_t)i].type = t;
      dims[(size_t)i].pad_ = 0;
      dims[(size_t)i].size = dim_sizes[(size_t)i];
      dims[(size_t)i].stride_left = strides[0][0][(size_t)i];
      dims[(size_t)i].stride_right = strides[0][1][(size_t)i];
      dims[(size_t)i].stride_out = strides[0][2][(size_t)i];
      dims[(size_t)i].stride_out_aux = 0;
    }
    eir_contract_desc desc{};
    desc.num_dims = nd;
    desc.dtype_left = desc.dtype_right = desc.dtype_out = dt;
    desc.dtype_comp = EIR_COMPUTE_DEFAULT;
    desc.ktype_first_touch = first;
    desc.ktype_main = EIR_KTYPE_MADD;
    desc.ktype_last_touch = last;
    desc.flags = 0;
    desc.dims = dims.data();
    if (eir_contract_plan_create(&desc, &plan) != EIR_SUCCESS) return error_t::compilation_failed;
  }
  m_plan = plan;
  m_op_type = op;
  return error_t::success;
}

void TensorOperation::execute(void const *tensor_in0, void const *tensor_in1, void *tensor_out) {
  if (m_op_type == op_type_t::unary)
    m_status = eir_permute(m_plan, tensor_in0, tensor_out, m_stream);
  else if (m_op_type == op_type_t::binary)
    m_status = eir_contract(m_plan, tensor_in0, tensor_in1, nullptr, tensor_out, m_stream);
  else
    m_status = EIR_CALLED_BEFORE_COMPILATION;
}

OptimizationConfig TensorOperation::get_default_optimization_config() {
  OptimizationConfig c;
  c.target_m = 16;
  c.target_n = 12;
  c.target_k = 64;
  c.num_threads = 0;
  c.packed_gemm_support = true;
  c.br_gemm_support = true;
  c.packing_support = true;
  c.sfc_support = true;
  c.l2_cache_size = 1048576;
  return c;
}

std::tuple<TO::error_t, TO::dtype_t, TO::prim_t, TO::prim_t, TO::prim_t, std::vector<TO::dim_t>,
           std::vector<TO::exec_t>, std::vector<int64_t>, TO::strides_t>
TensorOperation::optimize(dtype_t dtype, prim_t prim_first, prim_t prim_main, prim_t prim_last,
                          std::vector<dim_t> const &dim_types, std::vector<exec_t> const &exec_types,
                          std::vector<int64_t> const &dim_sizes, strides_t const &strides,
                          OptimizationConfig const &cfg) {
  auto fail = [&](error_t e) {
    return std::make_tuple(e, dtype, prim_first, prim_main, prim_last, dim_types, exec_types, dim_sizes,
                           strides_t());
  };
  const op_type_t op = op_type_of(prim_main);
  const error_t shape = check_level0(op, dim_sizes, strides);
  if (shape != error_t::success) return fail(shape);
  if (cfg.target_m < 0 || cfg.target_n < 0 || cfg.target_k < 0 || cfg.num_threads < 0 || cfg.l2_cache_size < 0)
    return fail(error_t::invalid_optimization_config);
  if (dim_types.size() != dim_sizes.size() || exec_types.size() != dim_sizes.size())
    return fail(error_t::compilation_failed);
  const bool binary = op == op_type_t::binary;
  const int tensors = binary ? 3 : 2;
  std::vector<LoopDim> d;
  for (size_t i = 0; i < dim_sizes.size(); ++i) {
    if (dim_sizes[i] <= 0 || (binary && eir_dim_type(dim_types[i]) < 0)) return fail(error_t::compilation_failed);
    LoopDim x;
    x.type = binary ? dim_types[i] : dim_t::c;
    x.size = dim_sizes[i];
    x.s[0] = strides[0][0][i];
    x.s[1] = strides[0][1][i];  // in1, or the output of a unary operation
    x.s[2] = binary ? strides[0][2][i] : 0;
    d.push_back(x);
  }
  d = simplify(d, tensors);
  std::vector<dim_t> types;
  std::vector<exec_t> execs;
  std::vector<int64_t> sizes;
  std::vector<int64_t> s0, s1, s2;
  // B200 execution: K loops inside a CTA (seq), C / M / N spread over CTAs
  // (shared); the tile dims of the kernel are prim: the output's fastest M
  // and N dims and the left operand's fastest K dim (unary: the output's
  // fastest dim, the vector access dim of the permute kernels)
  const int out_t = binary ? 2 : 1;
  const int pm = binary ? innermost(d, dim_t::m, out_t) : innermost(d, dim_t::c, out_t);
  const int pn = binary ? innermost(d, dim_t::n, out_t) : -1;
  const int pk = binary ? innermost(d, dim_t::k, 0) : -1;
  for (size_t i = 0; i < d.size(); ++i) {
    types.push_back(d[i].type);
    sizes.push_back(d[i].size);
    const int ii = (int)i;
    exec_t e = d[i].type == dim_t::k ? exec_t::seq : exec_t::shared;
    if (ii == pm || ii == pn || ii == pk) e = exec_t::prim;
    execs.push_back(e);
    s0.push_back(d[i].s[0]);
    s1.push_back(d[i].s[1]);
    s2.push_back(d[i].s[2]);
  }
  strides_t out_strides;
  if (binary) out_strides = {{s0, s1, s2}};
  else out_strides = {{s0, s1}};
  return std::make_tuple(error_t::success, dtype, prim_first, prim_main, prim_last, types, execs, sizes,
                         out_strides);
}

}  // namespace py
}  // namespace einsum_ir
