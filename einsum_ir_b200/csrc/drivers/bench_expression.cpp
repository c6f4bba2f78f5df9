// bench_expression: evaluates an einsum expression (contraction tree) on the
// GPU through the einsum_ir host classes and reports the reference driver's
// figures (#flops, compile / eval time, GFLOPS, CSV_DATA line) and a
// Frobenius relative-error check.
//
// Command line as the reference driver (src/bench_expression.cpp:8-31):
//   bench_expression einsum_string dimension_sizes contraction_path [dtype [store_lock [print_tree]]]
// dtype: FP32 (default), FP64, BF16 (BF16 inputs, FP32 accumulation and
// output), TF32 (FP32 data, single-pass TF32 tensor-core compute), CPX_FP32 or
// CPX_FP64 (complex, interleaved: a size-2 dim appended to every tensor as in
// src/bench_expression.cpp:110-247).
// Differences: data are seeded uniform [-1, 1) values (the reference draws
// at::randn); the eval time is the mean over a CUDA-event-timed loop (the
// reference times one eval with a host clock); the check solution is the
// same tree in FP64 on the CUDA-core kernels (the reference compares with
// at::einsum, src/bench_expression.cpp:380-541), with the reference's
// tolerances 1e-5 (FP32, BF16) and 1e-12 (FP64), 1e-2 for TF32. With
// EIR_DRIVER_DUMP=<dir> the inputs and the result are also written for the
// CPU oracle (see driver_util.h), which the tests compare against.
#include <cuda_runtime.h>
#include <chrono>
#include <cstdio>
#include <map>
#include <string>
#include <vector>
#include "BinaryContractionCuda.h"
#include "EinsumExpression.h"
#include "driver_util.h"
#include "eir_cuda.h"

using einsum_ir::frontend::EinsumExpression;
using einsum_ir::frontend::EinsumExpressionAscii;
using namespace eir_driver;

namespace {

void usage() {
  std::fprintf(stderr,
               "Usage:\n"
               "  ./bench_expression einsum_string dimension_sizes contraction_path dtype store_lock print_tree\n\n"
               "Arguments:\n"
               "  * einsum_string:    Einsum expression string. Either in single-character or standard format.\n"
               "  * dimension_sizes:  Dimension sizes have to be in ascending order of the dimension names.\n"
               "  * contraction_path: Contraction path.\n"
               "  * dtype:            FP32, FP64, BF16, TF32, CPX_FP32 or CPX_FP64, default: FP32.\n"
               "  * store_lock:       If 1 all input tensors are stored and locked before evaluation, default: 0.\n"
               "  * print_tree:       If not 0 the contraction tree is printed (1: dimension ids, 2: names), default: 0.\n\n"
               "Example:\n"
               "  ./bench_expression \"iae,bf,dcba,cg,dh->hgfei\" \"32,8,4,2,16,64,8,8,8\" \"(1,2),(2,3),(0,1),(0,1)\"\n");
}

struct Tree {
  std::vector<int64_t> string_num_dims, string_dim_ids, path, dim_sizes;
  int64_t num_tensors = 0;
  std::vector<std::vector<int64_t>> shapes;  // per tensor
};

std::string dims_string(std::vector<int64_t> const &ids, std::map<int64_t, std::string> const &names,
                        bool by_name) {
  std::string s = "[";
  for (size_t i = 0; i < ids.size(); ++i) {
    if (i) s += ",";
    s += by_name ? names.at(ids[i]) : std::to_string(ids[i]);
  }
  return s + "]";
}

void print_node(einsum_ir::backend::EinsumNode const &n, int depth,
                std::map<int64_t, std::string> const &names, bool by_name) {
  std::string pad(2 * depth, ' ');
  std::printf("%s%s", pad.c_str(), dims_string(n.m_dim_ids_int, names, by_name).c_str());
  if (n.m_cont != nullptr) {
    auto const *bc = static_cast<einsum_ir::backend::BinaryContractionCuda const *>(n.m_cont);
    std::printf("  <- %s", eir_plan_describe(bc->m_plan));
  }
  std::printf("\n");
  for (auto const *c : n.m_children) print_node(*c, depth + 1, names, by_name);
}

}  // namespace

int main(int argc, char *argv[]) {
  if (argc < 4) {
    usage();
    return EXIT_FAILURE;
  }
  // ---- expression, dimension ids and sizes (EinsumExpressionAscii as the reference driver)
  std::string expr_arg(argv[1]), expr_std, expr_schar;
  if (expr_arg[0] == '[') {
    expr_std = expr_arg;
    EinsumExpressionAscii::standard_to_schar(expr_std, expr_schar);
  } else {
    expr_schar = expr_arg;
    EinsumExpressionAscii::schar_to_standard(expr_schar, expr_std);
  }
  std::vector<std::string> tensors;
  EinsumExpressionAscii::parse_tensors(expr_std, tensors);
  std::printf("parsed tensors:\n");
  for (auto const &t : tensors) std::printf("  %s\n", t.c_str());

  std::map<std::string, int64_t> name_to_id;
  EinsumExpressionAscii::parse_dim_ids(expr_std, name_to_id);
  std::map<int64_t, std::string> id_to_name;
  std::printf("parsed dimension ids:\n");
  for (auto const &kv : name_to_id) {
    std::printf("  %s: %lld\n", kv.first.c_str(), (long long)kv.second);
    id_to_name[kv.second] = kv.first;
  }
  std::string sizes_arg(argv[2]);
  Tree tr;
  EinsumExpressionAscii::parse_dim_sizes(sizes_arg, tr.dim_sizes);
  if (tr.dim_sizes.size() != name_to_id.size()) {
    std::fprintf(stderr, "error: %zu dimension sizes for %zu dimensions\n", tr.dim_sizes.size(),
                 name_to_id.size());
    return EXIT_FAILURE;
  }
  std::printf("parsed dimension sizes:\n");
  for (auto const &kv : name_to_id)
    std::printf("  %s: %lld\n", kv.first.c_str(), (long long)tr.dim_sizes[kv.second]);
  std::string path_arg(argv[3]);
  EinsumExpressionAscii::parse_path(path_arg, tr.path);
  std::printf("parsed path:\n ");
  for (auto p : tr.path) std::printf(" %lld", (long long)p);
  std::printf("\n");

  std::string dtype = argc > 4 ? std::string(argv[4]) : std::string("FP32");
  einsum_ir::complex_t ctype = einsum_ir::UNDEFINED_CTYPE;
  EinsumExpressionAscii::parse_ctype(dtype, ctype);
  if (ctype == einsum_ir::UNDEFINED_CTYPE && dtype != "TF32") {
    std::fprintf(stderr, "failed to determine dtype\n");
    return EXIT_FAILURE;
  }
  const bool cpx = ctype == einsum_ir::BATCH_INNER;
  std::printf("dtype: %s\n", dtype.c_str());
  std::printf("ctype: %s\n", cpx ? "BATCH_INNER" : "REAL_ONLY");
  // complex: one more dim (size 2, the largest id) innermost in every tensor
  const int64_t cpx_id = (int64_t)name_to_id.size();
  if (cpx) {
    tr.dim_sizes.push_back(2);
    id_to_name[cpx_id] = "(cpx)";
  }
  const bool store_lock = argc > 5 && std::stoi(argv[5]) == 1;
  std::printf("store_lock: %d\n", store_lock ? 1 : 0);
  const int print_tree = argc > 6 ? std::stoi(argv[6]) : 0;
  if (print_tree < 0 || print_tree > 2) {
    std::fprintf(stderr, "error: invalid print_tree argument\n");
    return EXIT_FAILURE;
  }
  std::printf("print_tree: %d\n", print_tree);

  tr.num_tensors = (int64_t)tensors.size();
  if (tr.num_tensors < 3 || (int64_t)tr.path.size() != 2 * (tr.num_tensors - 2)) {
    std::fprintf(stderr, "error: the path needs one pair per contraction\n");
    return EXIT_FAILURE;
  }
  for (auto const &t : tensors) {
    std::vector<std::string> names;
    EinsumExpressionAscii::split_string(t, ",", names);
    std::vector<int64_t> shape;
    for (auto const &n : names) {
      tr.string_dim_ids.push_back(name_to_id[n]);
      shape.push_back(tr.dim_sizes[name_to_id[n]]);
    }
    if (cpx) {
      tr.string_dim_ids.push_back(cpx_id);
      shape.push_back(2);
    }
    tr.string_num_dims.push_back((int64_t)names.size() + (cpx ? 1 : 0));
    tr.shapes.push_back(shape);
  }

  // ---- data: seeded uniform inputs, stored in the run's input type
  const bool fp64 = dtype == "FP64" || dtype == "CPX_FP64";
  const int in_esize = fp64 ? 8 : (dtype == "BF16" ? 2 : 4);
  const int out_esize = fp64 ? 8 : 4;
  const einsum_ir::data_t dt = fp64 ? einsum_ir::FP64 : einsum_ir::FP32;
  std::vector<DeviceTensor> dev(tr.num_tensors);
  std::vector<std::vector<double>> held(tr.num_tensors);
  std::vector<void *> ptrs(tr.num_tensors);
  for (int64_t t = 0; t < tr.num_tensors; ++t) {
    int64_t n = 1;
    for (auto s : tr.shapes[t]) n *= s;
    bool is_out = t + 1 == tr.num_tensors;
    auto v = is_out ? std::vector<double>((size_t)n, 0.0) : uniform(n, 1234 + (uint64_t)t);
    held[t] = upload(v, is_out ? out_esize : in_esize, dev[t]);
    ptrs[t] = dev[t].ptr;
  }
  cudaStream_t st;
  check_cuda(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate");

  // ---- einsum_ir on the GPU
  std::printf("\n*** benchmarking einsum_ir (B200) ***\n");
  EinsumExpression exp;
  if (dtype == "BF16") exp.set_input_dtype(einsum_ir::BF16);
  if (dtype == "TF32") exp.set_compute_type(EIR_COMPUTE_TF32);
  exp.init((int64_t)tr.dim_sizes.size(), tr.dim_sizes.data(), tr.num_tensors - 2,
           tr.string_num_dims.data(), tr.string_dim_ids.data(), tr.path.data(),
           cpx ? einsum_ir::BATCH_INNER : einsum_ir::REAL_ONLY, dt, ptrs.data());
  exp.set_stream(st);
  auto tp0 = std::chrono::steady_clock::now();
  einsum_ir::err_t err = exp.compile();
  auto tp1 = std::chrono::steady_clock::now();
  const double t_compile = std::chrono::duration<double>(tp1 - tp0).count();
  if (err != einsum_ir::SUCCESS) {
    std::fprintf(stderr, "error: failed to compile einsum_ir expression (%d): %s\n", (int)err,
                 eir_last_error_string());
    return EXIT_FAILURE;
  }
  if (print_tree != 0) print_node(exp.nodes().back(), 0, id_to_name, print_tree == 2);
  if (store_lock) {
    for (int64_t t = 0; t + 1 < tr.num_tensors; ++t) {
      if (exp.store_and_lock_data(t) != einsum_ir::SUCCESS) {
        std::fprintf(stderr, "error: failed to store and lock tensor with id: %lld\n", (long long)t);
        return EXIT_FAILURE;
      }
    }
  }
  int rc = EIR_SUCCESS;
  const double t_eval = time_calls([&] { rc |= exp.eval(); }, st);
  check_cuda(cudaStreamSynchronize(st), "eval");
  if (rc != EIR_SUCCESS || eir_check_device_errors(st) != EIR_SUCCESS) {
    std::fprintf(stderr, "error: eval failed: %s\n", eir_last_error_string());
    return EXIT_FAILURE;
  }
  const int64_t flops = exp.num_ops();
  const double gf_eval = 1e-9 * (double)flops / t_eval;
  const double gf_total = 1e-9 * (double)flops / (t_compile + t_eval);
  std::printf("  #flops:         %lld\n", (long long)flops);
  std::printf("  time (compile): %g\n", t_compile);
  std::printf("  time (eval):    %g\n", t_eval);
  std::printf("  gflops (eval):  %g\n", gf_eval);
  std::printf("  gflops (total): %g\n", gf_total);
  std::printf("CSV_DATA: einsum_ir_b200,\"%s\",\"%s\",\"%s\",%lld,%g,%g,%g,%g\n", expr_arg.c_str(),
              sizes_arg.c_str(), path_arg.c_str(), (long long)flops, t_compile, t_eval, gf_eval,
              gf_total);

  // ---- C M N K of the binary contractions (the reference's at::matmul section)
  std::printf("  C M N K for the binary contractions:\n");
  auto &nodes = exp.nodes();
  for (int64_t c = 0; c + 2 < tr.num_tensors; ++c) {
    auto const *bc = nodes[tr.num_tensors - 1 + c].m_cont;
    int64_t s[4] = {1, 1, 1, 1};
    for (auto x : bc->m_sizes_c) s[0] *= x;
    for (auto x : bc->m_sizes_m) s[1] *= x;
    for (auto x : bc->m_sizes_n) s[2] *= x;
    for (auto x : bc->m_sizes_k) s[3] *= x;
    std::printf("    #%lld: %lld %lld %lld %lld\n", (long long)c, (long long)s[0], (long long)s[1],
                (long long)s[2], (long long)s[3]);
  }

  // ---- check: the same tree in FP64 on the CUDA-core kernels, same input values
  std::vector<double> got = download(dev.back());
  {
    Dump dump;  // EIR_DRIVER_DUMP: inputs and result for the CPU oracle
    dump.line("expr", expr_arg);
    dump.line("sizes", sizes_arg);
    dump.line("path", path_arg);
    dump.line("dtype", dtype);
    for (int64_t t = 0; t < tr.num_tensors; ++t) {
      std::vector<int64_t> tids;
      int64_t off = 0;
      for (int64_t u = 0; u < t; ++u) off += tr.string_num_dims[u];
      for (int64_t d = 0; d < tr.string_num_dims[t]; ++d) tids.push_back(tr.string_dim_ids[off + d]);
      const bool is_out = t + 1 == tr.num_tensors;
      dump.tensor(is_out ? "out" : "in" + std::to_string(t), tids, tr.shapes[t], is_out ? got : held[t]);
    }
  }
  std::vector<DeviceTensor> ref_dev(tr.num_tensors);
  std::vector<void *> ref_ptrs(tr.num_tensors);
  for (int64_t t = 0; t < tr.num_tensors; ++t) {
    upload(held[t], 8, ref_dev[t]);
    ref_ptrs[t] = ref_dev[t].ptr;
  }
  std::vector<double> ref;
  {
    CudaCoreOnly guard;
    EinsumExpression ref_exp;
    ref_exp.init((int64_t)tr.dim_sizes.size(), tr.dim_sizes.data(), tr.num_tensors - 2,
                 tr.string_num_dims.data(), tr.string_dim_ids.data(), tr.path.data(),
                 cpx ? einsum_ir::BATCH_INNER : einsum_ir::REAL_ONLY, einsum_ir::FP64, ref_ptrs.data());
    ref_exp.set_stream(st);
    if (ref_exp.compile() != einsum_ir::SUCCESS || ref_exp.eval() != EIR_SUCCESS) {
      std::fprintf(stderr, "error: FP64 check solution failed: %s\n", eir_last_error_string());
      return EXIT_FAILURE;
    }
    check_cuda(cudaStreamSynchronize(st), "check solution");
    ref = download(ref_dev.back());
  }
  std::printf("\n*** comparing solution ***:\n");
  ErrorReport r = compare(ref, got);
  print_report(r, "FP64 CUDA-core solution");
  const double tol = fp64 ? 1e-12 : (dtype == "TF32" ? 1e-2 : 1e-5);
  cudaStreamDestroy(st);
  if (r.rel > tol) {
    std::fprintf(stderr, "warning: relative error is large!\n");
    return EXIT_FAILURE;
  }
  return EXIT_SUCCESS;
}
