// bench_tree: evaluates a pre-optimised einsum tree string on the GPU through
// EinsumTree / EinsumTreeAscii, as the reference driver src/bench_tree.cpp
// does on the CPU, and checks the result against the same tree in FP64 on
// the CUDA-core kernels.
//
//   bench_tree einsum_tree dimension_sizes [dtype]
// dtype: FP32 (default), FP64, BF16 (BF16 leaves, FP32 inner nodes and output)
// or TF32. Data: seeded uniform [-1, 1) leaves (the reference draws
// at::randn); eval time: mean of a CUDA-event-timed loop. With
// EIR_DRIVER_DUMP=<dir> the parsed tree, the leaves and the result are also
// written for the CPU oracle (see driver_util.h).
#include <cuda_runtime.h>
#include <chrono>
#include <cstdio>
#include <map>
#include <string>
#include <vector>
#include "EinsumTree.h"
#include "driver_util.h"
#include "eir_cuda.h"

using einsum_ir::frontend::EinsumTree;
using einsum_ir::frontend::EinsumTreeAscii;
using namespace eir_driver;

namespace {

// evaluates the parsed tree once on `st` with the given data pointers
einsum_ir::err_t build(EinsumTree &tree, std::vector<std::vector<int64_t>> &ids,
                       std::vector<std::vector<int64_t>> &children, std::map<int64_t, int64_t> &sizes,
                       std::string const &dtype, std::vector<void *> const &ptrs, cudaStream_t st) {
  const einsum_ir::data_t dt = dtype == "FP64" ? einsum_ir::FP64 : einsum_ir::FP32;
  if (dtype == "BF16") tree.set_input_dtype(einsum_ir::BF16);
  if (dtype == "TF32") tree.set_compute_type(EIR_COMPUTE_TF32);
  tree.set_stream(st);
  tree.init(&ids, &children, &sizes, dt, ptrs.data());
  return tree.compile();
}

}  // namespace

int main(int argc, char *argv[]) {
  if (argc < 3) {
    std::fprintf(stderr,
                 "Usage:\n"
                 "  ./bench_tree einsum_tree dimension_sizes dtype\n\n"
                 "Arguments:\n"
                 "  * einsum_tree:      A compiled einsum tree.\n"
                 "  * dimension_sizes:  Dimension sizes have to be in ascending order of the dimension ids.\n"
                 "  * dtype:            FP32, FP64, BF16 or TF32, default: FP32.\n\n"
                 "Example:\n"
                 "  ./bench_tree \"[[3,0]->[0,3]],[[3,2,4],[1,4,2]->[1,2,3]]->[0,1,2]\" \"2,3,4,5,6\" FP32\n");
    return EXIT_FAILURE;
  }
  std::string tree_arg(argv[1]), sizes_arg(argv[2]);
  std::string dtype = argc > 3 ? std::string(argv[3]) : std::string("FP32");
  if (dtype != "FP32" && dtype != "FP64" && dtype != "BF16" && dtype != "TF32") {
    std::fprintf(stderr, "failed to determine dtype\n");
    return EXIT_FAILURE;
  }
  const int64_t n = EinsumTreeAscii::count_nodes(tree_arg);
  std::vector<std::vector<int64_t>> ids(n), children(n);
  int64_t parsed = 0;
  if (EinsumTreeAscii::parse_tree(tree_arg, ids, children, parsed) != einsum_ir::SUCCESS || parsed != n) {
    std::fprintf(stderr, "error: failed to parse einsum tree\n");
    return EXIT_FAILURE;
  }
  std::map<int64_t, int64_t> sizes;
  EinsumTreeAscii::parse_dim_size(sizes_arg, ids, sizes);
  for (auto const &t : ids)
    for (auto d : t)
      if (!sizes.count(d)) {
        std::fprintf(stderr, "error: no size for dimension %lld\n", (long long)d);
        return EXIT_FAILURE;
      }
  std::printf("nodes: %lld, dtype: %s\n", (long long)n, dtype.c_str());

  // external tensors: leaves and the root
  const int in_esize = dtype == "FP64" ? 8 : (dtype == "BF16" ? 2 : 4);
  const int out_esize = dtype == "FP64" ? 8 : 4;
  std::vector<DeviceTensor> dev(n), ref_dev(n);
  std::vector<void *> ptrs(n, nullptr), ref_ptrs(n, nullptr);
  for (int64_t i = 0; i < n; ++i) {
    const bool root = i + 1 == n;
    if (!children[i].empty() && !root) continue;
    int64_t count = 1;
    for (auto d : ids[i]) count *= sizes[d];
    auto v = root ? std::vector<double>((size_t)count, 0.0) : uniform(count, 99 + (uint64_t)i);
    auto held = upload(v, root ? out_esize : in_esize, dev[i]);
    upload(held, 8, ref_dev[i]);
    ptrs[i] = dev[i].ptr;
    ref_ptrs[i] = ref_dev[i].ptr;
  }
  cudaStream_t st;
  check_cuda(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate");

  std::printf("\n*** benchmarking einsum_ir (B200) ***\n");
  EinsumTree tree;
  auto tp0 = std::chrono::steady_clock::now();
  einsum_ir::err_t err = build(tree, ids, children, sizes, dtype, ptrs, st);
  auto tp1 = std::chrono::steady_clock::now();
  if (err != einsum_ir::SUCCESS) {
    std::fprintf(stderr, "error: failed to compile einsum_ir tree (%d): %s\n", (int)err,
                 eir_last_error_string());
    return EXIT_FAILURE;
  }
  const double t_compile = std::chrono::duration<double>(tp1 - tp0).count();
  int rc = EIR_SUCCESS;
  const double t_eval = time_calls([&] { rc |= tree.eval(); }, st);
  if (rc != EIR_SUCCESS || eir_check_device_errors(st) != EIR_SUCCESS) {
    std::fprintf(stderr, "error: eval failed: %s\n", eir_last_error_string());
    return EXIT_FAILURE;
  }
  const int64_t flops = tree.num_ops();
  const double gf_eval = 1e-9 * (double)flops / t_eval;
  const double gf_total = 1e-9 * (double)flops / (t_compile + t_eval);
  std::printf("  #flops:         %lld\n", (long long)flops);
  std::printf("  time (compile): %g\n", t_compile);
  std::printf("  time (eval):    %g\n", t_eval);
  std::printf("  gflops (eval):  %g\n", gf_eval);
  std::printf("  gflops (total): %g\n", gf_total);
  std::printf("CSV_DATA: einsum_ir_b200,\"%s\",\"%s\",%lld,%g,%g,%g,%g\n", tree_arg.c_str(),
              sizes_arg.c_str(), (long long)flops, t_compile, t_eval, gf_eval, gf_total);

  std::vector<double> got = download(dev[n - 1]), ref;
  {
    Dump dump;  // EIR_DRIVER_DUMP: the parsed tree, its leaves and the result for the CPU oracle
    dump.line("tree", tree_arg);
    dump.line("sizes", sizes_arg);
    dump.line("dtype", dtype);
    for (int64_t i = 0; i < n; ++i) {
      std::string ch;
      for (size_t c = 0; c < children[i].size(); ++c) ch += (c ? "," : "") + std::to_string(children[i][c]);
      std::string ids_s;
      for (size_t d = 0; d < ids[i].size(); ++d) ids_s += (d ? "," : "") + std::to_string(ids[i][d]);
      dump.line("node" + std::to_string(i),
                "ids " + (ids_s.empty() ? "-" : ids_s) + " children " + (ch.empty() ? "-" : ch));
      std::vector<int64_t> shp;
      for (auto d : ids[i]) shp.push_back(sizes[d]);
      if (i + 1 == n) dump.tensor("out", ids[i], shp, got);
      else if (children[i].empty()) dump.tensor("leaf" + std::to_string(i), ids[i], shp, download(ref_dev[i]));
    }
  }
  {
    CudaCoreOnly guard;
    EinsumTree ref_tree;
    if (build(ref_tree, ids, children, sizes, "FP64", ref_ptrs, st) != einsum_ir::SUCCESS ||
        ref_tree.eval() != EIR_SUCCESS) {
      std::fprintf(stderr, "error: FP64 check solution failed: %s\n", eir_last_error_string());
      return EXIT_FAILURE;
    }
    check_cuda(cudaStreamSynchronize(st), "check solution");
    ref = download(ref_dev[n - 1]);
  }
  std::printf("\n*** comparing solution ***:\n");
  ErrorReport r = compare(ref, got);
  print_report(r, "FP64 CUDA-core solution");
  cudaStreamDestroy(st);
  const double tol = dtype == "FP64" ? 1e-12 : (dtype == "TF32" ? 1e-2 : 1e-5);
  if (r.rel > tol) {
    std::fprintf(stderr, "warning: relative error is large!\n");
    return EXIT_FAILURE;
  }
  return EXIT_SUCCESS;
}
