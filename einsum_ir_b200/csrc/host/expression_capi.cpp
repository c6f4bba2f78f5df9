// C-ABI of einsum expressions (eir_expression_*): string parsing as in the
// reference's bench_expression driver (src/bench_expression.cpp:35-189), tree
// compilation through frontend::EinsumExpression, evaluation on a stream.
//
// Evaluation of a whole tree is launch-latency bound for small trees, so on a
// non-default stream the tree is captured into a CUDA graph once it has run
// eagerly with a given set of data pointers (the eager run performs every
// lazy allocation), and later calls with the same pointers and stream replay
// the graph. EIR_EXPRESSION_GRAPHS=0 disables this.
#include <cuda_runtime.h>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <map>
#include <string>
#include <vector>
#include "BinaryContractionCuda.h"
#include "EinsumExpression.h"
#include "eir_cuda.h"

namespace eir {
int api_set_error(int code, char const *msg);  // eir_capi.cu: shared last-error string
}

using einsum_ir::frontend::EinsumExpression;
using einsum_ir::frontend::EinsumExpressionAscii;

struct eir_expression {
  EinsumExpression expr;
  std::vector<int64_t> dim_sizes;
  std::vector<int64_t> string_num_dims;
  std::vector<int64_t> string_dim_ids;
  std::vector<int64_t> path;
  std::vector<void *> sentinel_ptrs;
  int64_t num_tensors = 0;
  std::string text;
  // graph replay state
  std::vector<void *> last_ptrs;
  void *last_stream = nullptr;
  int eager_runs = 0;
  cudaGraphExec_t graph = nullptr;
};

namespace {
int fail(int code, std::string const &msg) { return eir::api_set_error(code, msg.c_str()); }
bool graphs_enabled() {
  char const *v = std::getenv("EIR_EXPRESSION_GRAPHS");
  return v == nullptr || std::strcmp(v, "0") != 0;
}
}  // namespace

extern "C" {

int eir_expression_create(char const *expr_str, char const *sizes_str, char const *path_str,
                          int32_t dtype, int32_t dtype_comp, eir_expression **out) {
  if (out == nullptr || expr_str == nullptr || sizes_str == nullptr)
    return fail(EIR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  if (dtype != EIR_FP32 && dtype != EIR_FP64 && dtype != EIR_BF16)
    return fail(EIR_INVALID_DTYPE, "unsupported dtype");
  auto *e = new eir_expression();
  try {
    std::string expr(expr_str), standard;
    if (expr.find('[') == std::string::npos) EinsumExpressionAscii::schar_to_standard(expr, standard);
    else standard = expr;
    std::vector<std::string> tensors;
    EinsumExpressionAscii::parse_tensors(standard, tensors);
    std::map<std::string, int64_t> ids;
    EinsumExpressionAscii::parse_dim_ids(standard, ids);
    for (auto const &t : tensors) {
      std::vector<std::string> dims;
      EinsumExpressionAscii::split_string(t, ",", dims);
      e->string_num_dims.push_back((int64_t)dims.size());
      for (auto const &d : dims) e->string_dim_ids.push_back(ids.at(d));
    }
    EinsumExpressionAscii::parse_dim_sizes(sizes_str, e->dim_sizes);
    if (e->dim_sizes.size() != ids.size()) {
      delete e;
      return fail(EIR_INVALID_ARGUMENT, "number of sizes does not match the number of dims");
    }
    const int64_t n_in = (int64_t)tensors.size() - 1;
    if (n_in < 2) {
      delete e;
      return fail(EIR_INVALID_ARGUMENT, "an expression needs at least two input tensors");
    }
    if (path_str != nullptr && std::strlen(path_str) > 0) EinsumExpressionAscii::parse_path(path_str, e->path);
    else
      for (int64_t c = 0; c < n_in - 1; ++c) {  // default: always contract the first two
        e->path.push_back(0);
        e->path.push_back(1);
      }
    if ((int64_t)e->path.size() != 2 * (n_in - 1)) {
      delete e;
      return fail(EIR_INVALID_ARGUMENT, "path must have one pair per contraction");
    }
    e->num_tensors = n_in + 1;
    // non-null placeholders: inputs and output are external tensors; the real
    // device pointers are bound at every eval
    e->sentinel_ptrs.assign(e->num_tensors, reinterpret_cast<void *>(uintptr_t(256)));
    einsum_ir::data_t dt = dtype == EIR_FP64 ? einsum_ir::FP64 : einsum_ir::FP32;
    e->expr.set_input_dtype(dtype == EIR_BF16 ? einsum_ir::BF16 : dt);
    e->expr.set_compute_type(dtype_comp);
    e->expr.init((int64_t)e->dim_sizes.size(), e->dim_sizes.data(), n_in - 1,
                 e->string_num_dims.data(), e->string_dim_ids.data(), e->path.data(), dt,
                 e->sentinel_ptrs.data());
    einsum_ir::err_t err = e->expr.compile();
    if (err != einsum_ir::SUCCESS) {
      delete e;
      return fail((int)err, "expression compile failed (err_t " + std::to_string((int)err) + ")");
    }
  } catch (std::exception const &ex) {
    delete e;
    return fail(EIR_INVALID_ARGUMENT, std::string("cannot parse expression: ") + ex.what());
  }
  e->text = std::string(expr_str);
  *out = e;
  return EIR_SUCCESS;
}

int eir_expression_eval(eir_expression *e, void *const *ptrs, void *stream) {
  if (e == nullptr || ptrs == nullptr) return fail(EIR_INVALID_ARGUMENT, "null argument");
  for (int64_t t = 0; t < e->num_tensors; ++t)
    if (ptrs[t] == nullptr) return fail(EIR_NO_DATA_PTR_PROVIDED, "null tensor pointer");
  std::vector<void *> p(ptrs, ptrs + e->num_tensors);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  bool same = p == e->last_ptrs && stream == e->last_stream;
  if (!same) {
    if (e->graph) cudaGraphExecDestroy(e->graph);
    e->graph = nullptr;
    e->eager_runs = 0;
    e->last_ptrs = p;
    e->last_stream = stream;
  }
  e->expr.set_data_ptrs(ptrs);
  e->expr.set_stream(stream);
  if (e->graph != nullptr) {
    cudaError_t ce = cudaGraphLaunch(e->graph, st);
    return ce == cudaSuccess ? EIR_SUCCESS : fail(EIR_CUDA_ERROR, cudaGetErrorString(ce));
  }
  bool capture = graphs_enabled() && stream != nullptr && e->eager_runs >= 1;
  if (capture) {
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
      int rc = e->expr.eval();
      cudaError_t ce = cudaStreamEndCapture(st, &g);
      if (rc == EIR_SUCCESS && ce == cudaSuccess && g != nullptr &&
          cudaGraphInstantiate(&e->graph, g, 0) == cudaSuccess) {
        cudaGraphDestroy(g);
        cudaError_t le = cudaGraphLaunch(e->graph, st);
        return le == cudaSuccess ? EIR_SUCCESS : fail(EIR_CUDA_ERROR, cudaGetErrorString(le));
      }
      if (g != nullptr) cudaGraphDestroy(g);
      e->graph = nullptr;
      cudaGetLastError();  // clear a capture error and fall back to eager launches
    }
  }
  int rc = e->expr.eval();
  e->eager_runs++;
  if (rc != EIR_SUCCESS) return rc;  // the failing call set the error string
  return EIR_SUCCESS;
}

int64_t eir_expression_num_ops(eir_expression const *e) {
  return e == nullptr ? 0 : const_cast<eir_expression *>(e)->expr.num_ops();
}

int eir_expression_num_tensors(eir_expression const *e) { return e ? (int)e->num_tensors : 0; }

int eir_expression_tensor_dims(eir_expression const *e, int32_t tensor, int64_t *sizes_out,
                               int32_t max_dims) {
  if (e == nullptr || tensor < 0 || tensor >= e->num_tensors) return -EIR_INVALID_ID;
  int64_t off = 0;
  for (int32_t t = 0; t < tensor; ++t) off += e->string_num_dims[t];
  int64_t n = e->string_num_dims[tensor];
  if (n > max_dims) return -EIR_INVALID_ARGUMENT;
  for (int64_t d = 0; d < n; ++d) sizes_out[d] = e->dim_sizes[e->string_dim_ids[off + d]];
  return (int)n;
}

int eir_expression_destroy(eir_expression *e) {
  if (e == nullptr) return EIR_SUCCESS;
  if (e->graph) cudaGraphExecDestroy(e->graph);
  delete e;
  return EIR_SUCCESS;
}

char const *eir_expression_describe(eir_expression const *e) {
  if (e == nullptr) return "";
  auto *me = const_cast<eir_expression *>(e);
  std::string s;
  for (auto &n : me->expr.nodes()) {
    if (n.m_children.size() != 2) continue;
    auto ids = [](einsum_ir::backend::EinsumNode const *x) {
      std::string r;
      for (int64_t d = 0; d < x->m_num_dims; ++d) r += (d ? "," : "") + std::to_string(x->m_dim_ids_int[d]);
      return "[" + r + "]";
    };
    s += ids(n.m_children[0]) + " x " + ids(n.m_children[1]) + " -> " + ids(&n) + " : ";
    auto *bc = static_cast<einsum_ir::backend::BinaryContractionCuda *>(n.m_cont);
    s += bc->m_plan ? eir_plan_describe(bc->m_plan) : "(no plan)";
    s += "\n";
  }
  me->text = s;
  return me->text.c_str();
}

}  // extern "C"
