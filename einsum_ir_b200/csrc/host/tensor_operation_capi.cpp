// C-ABI of TensorOperation (eir_top_*): flattened descriptors in, the
// reference's error_t values out (see eir_tensor_operation.h).
#include <exception>
#include <vector>
#include "TensorOperation.h"
#include "eir_tensor_operation.h"

namespace eir {
int api_set_error(int code, char const *msg);  // eir_capi.cu: shared last-error string
}

using einsum_ir::py::OptimizationConfig;
using einsum_ir::py::TensorOperation;

struct eir_tensor_operation {
  TensorOperation op;
};

namespace {

constexpr int kErr = (int)TensorOperation::error_t::compilation_failed;
constexpr int kShape = (int)TensorOperation::error_t::invalid_stride_shape;

bool valid_enum(int32_t v, int32_t hi) { return v >= 0 && v <= hi; }

// unflattens [LEVEL][TENSOR][DIMENSION]; false on negative counts
bool unflatten(int32_t num_levels, int32_t const *tensors_per_level, int32_t const *dims_per_vector,
               int64_t const *strides, TensorOperation::strides_t *out) {
  out->clear();
  if (num_levels < 0) return false;
  if (num_levels > 0 && tensors_per_level == nullptr) return false;
  size_t v = 0, pos = 0;
  for (int32_t l = 0; l < num_levels; ++l) {
    if (tensors_per_level[l] < 0) return false;
    std::vector<std::vector<int64_t>> level;
    for (int32_t t = 0; t < tensors_per_level[l]; ++t, ++v) {
      if (dims_per_vector == nullptr || dims_per_vector[v] < 0) return false;
      std::vector<int64_t> vec((size_t)dims_per_vector[v]);
      for (auto &x : vec) {
        if (strides == nullptr) return false;
        x = strides[pos++];
      }
      level.push_back(std::move(vec));
    }
    out->push_back(std::move(level));
  }
  return true;
}

// enum vectors of one descriptor; false on out-of-range values
bool descriptor(int32_t num_dims, int32_t const *dim_types, int32_t const *exec_types,
                int64_t const *dim_sizes, std::vector<TensorOperation::dim_t> *dt,
                std::vector<TensorOperation::exec_t> *et, std::vector<int64_t> *ds) {
  if (num_dims < 0 || (num_dims > 0 && (dim_types == nullptr || exec_types == nullptr || dim_sizes == nullptr)))
    return false;
  for (int32_t i = 0; i < num_dims; ++i) {
    if (!valid_enum(dim_types[i], 3) || !valid_enum(exec_types[i], 3)) return false;
    dt->push_back((TensorOperation::dim_t)dim_types[i]);
    et->push_back((TensorOperation::exec_t)exec_types[i]);
    ds->push_back(dim_sizes[i]);
  }
  return true;
}

bool prims(int32_t dtype, int32_t a, int32_t b, int32_t c) {
  return valid_enum(dtype, 1) && valid_enum(a, 5) && valid_enum(b, 5) && valid_enum(c, 5);
}

}  // namespace

extern "C" {

int eir_top_create(eir_tensor_operation **op) {
  if (op == nullptr) return eir::api_set_error(EIR_INVALID_ARGUMENT, "null argument");
  try {
    *op = new eir_tensor_operation();
  } catch (std::exception const &) {
    return eir::api_set_error(EIR_UNDEFINED_ERROR, "allocation failed");
  }
  return EIR_SUCCESS;
}

int eir_top_destroy(eir_tensor_operation *op) {
  delete op;
  return EIR_SUCCESS;
}

int eir_top_setup(eir_tensor_operation *op, int32_t dtype, int32_t prim_first, int32_t prim_main,
                  int32_t prim_last, int32_t num_dims, int32_t const *dim_types,
                  int32_t const *exec_types, int64_t const *dim_sizes, int32_t num_levels,
                  int32_t const *tensors_per_level, int32_t const *dims_per_vector,
                  int64_t const *strides) {
  if (op == nullptr) return kErr;
  try {
    std::vector<TensorOperation::dim_t> dt;
    std::vector<TensorOperation::exec_t> et;
    std::vector<int64_t> ds;
    TensorOperation::strides_t st;
    if (!prims(dtype, prim_first, prim_main, prim_last)) return kErr;
    if (!descriptor(num_dims, dim_types, exec_types, dim_sizes, &dt, &et, &ds)) return kErr;
    if (!unflatten(num_levels, tensors_per_level, dims_per_vector, strides, &st)) return kShape;
    return (int)op->op.setup((TensorOperation::dtype_t)dtype, (TensorOperation::prim_t)prim_first,
                             (TensorOperation::prim_t)prim_main, (TensorOperation::prim_t)prim_last, dt, et,
                             ds, st);
  } catch (std::exception const &) {
    return kErr;
  }
}

int eir_top_execute(eir_tensor_operation *op, void const *in0, void const *in1, void *out, void *stream) {
  if (op == nullptr) return eir::api_set_error(EIR_INVALID_ARGUMENT, "null operation");
  op->op.set_stream(stream);
  op->op.execute(in0, in1, out);
  return op->op.last_status();
}

eir_plan const *eir_top_plan(eir_tensor_operation const *op) { return op == nullptr ? nullptr : op->op.plan(); }

int eir_top_default_optimization_config(eir_top_optimization_config *cfg) {
  if (cfg == nullptr) return eir::api_set_error(EIR_INVALID_ARGUMENT, "null argument");
  OptimizationConfig c = TensorOperation::get_default_optimization_config();
  cfg->target_m = c.target_m;
  cfg->target_n = c.target_n;
  cfg->target_k = c.target_k;
  cfg->num_threads = c.num_threads;
  cfg->br_gemm_support = c.br_gemm_support;
  cfg->packed_gemm_support = c.packed_gemm_support;
  cfg->packing_support = c.packing_support;
  cfg->sfc_support = c.sfc_support;
  cfg->l2_cache_size = c.l2_cache_size;
  return EIR_SUCCESS;
}

int eir_top_optimize(int32_t dtype, int32_t prim_first, int32_t prim_main, int32_t prim_last,
                     int32_t num_dims, int32_t const *dim_types, int32_t const *exec_types,
                     int64_t const *dim_sizes, int32_t num_levels, int32_t const *tensors_per_level,
                     int32_t const *dims_per_vector, int64_t const *strides,
                     eir_top_optimization_config const *cfg, int32_t *out_num_dims,
                     int32_t *out_dim_types, int32_t *out_exec_types, int64_t *out_dim_sizes,
                     int32_t *out_tensors, int64_t *out_strides) {
  if (cfg == nullptr || out_num_dims == nullptr || out_tensors == nullptr) return kErr;
  try {
    std::vector<TensorOperation::dim_t> dt;
    std::vector<TensorOperation::exec_t> et;
    std::vector<int64_t> ds;
    TensorOperation::strides_t st;
    if (!prims(dtype, prim_first, prim_main, prim_last)) return kErr;
    if (!descriptor(num_dims, dim_types, exec_types, dim_sizes, &dt, &et, &ds)) return kErr;
    if (!unflatten(num_levels, tensors_per_level, dims_per_vector, strides, &st)) return kShape;
    OptimizationConfig c;
    c.target_m = cfg->target_m;
    c.target_n = cfg->target_n;
    c.target_k = cfg->target_k;
    c.num_threads = cfg->num_threads;
    c.br_gemm_support = cfg->br_gemm_support != 0;
    c.packed_gemm_support = cfg->packed_gemm_support != 0;
    c.packing_support = cfg->packing_support != 0;
    c.sfc_support = cfg->sfc_support != 0;
    c.l2_cache_size = cfg->l2_cache_size;
    auto r = TensorOperation::optimize((TensorOperation::dtype_t)dtype, (TensorOperation::prim_t)prim_first,
                                       (TensorOperation::prim_t)prim_main, (TensorOperation::prim_t)prim_last,
                                       dt, et, ds, st, c);
    const auto err = std::get<0>(r);
    if (err != TensorOperation::error_t::success) return (int)err;
    auto const &odt = std::get<5>(r);
    auto const &oet = std::get<6>(r);
    auto const &ods = std::get<7>(r);
    auto const &ost = std::get<8>(r);
    if ((int32_t)ods.size() > num_dims || out_dim_types == nullptr || out_exec_types == nullptr ||
        out_dim_sizes == nullptr || out_strides == nullptr)
      return kErr;
    *out_num_dims = (int32_t)ods.size();
    *out_tensors = (int32_t)ost[0].size();
    for (size_t i = 0; i < ods.size(); ++i) {
      out_dim_types[i] = (int32_t)odt[i];
      out_exec_types[i] = (int32_t)oet[i];
      out_dim_sizes[i] = ods[i];
    }
    size_t pos = 0;
    for (auto const &v : ost[0])
      for (int64_t x : v) out_strides[pos++] = x;
    return (int)err;
  } catch (std::exception const &) {
    return kErr;
  }
}

}  // extern "C"
