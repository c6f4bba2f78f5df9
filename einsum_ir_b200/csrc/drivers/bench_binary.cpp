// bench_binary: one strided binary contraction through BinaryContractionCuda
// (no EinsumNode: no swap, no reorder, no unary), as the reference driver
// src/bench_binary.cpp:12-408 does with BinaryContractionTpp.
//
//   bench_binary einsum_string dimension_sizes [dtype [loop_order]]
// dtype: FP32 (default), FP64, BF16 (BF16 inputs, FP32 output) or TF32.
// loop_order is accepted and printed; the GPU backend chooses its own tiling.
// Data as the reference driver: left uniform [0, 1), right ones (:57-59).
// Timing: repeated contract() calls for ~0.5 s with CUDA events. Check: the
// same contraction in FP64 on the CUDA-core kernel, relative Frobenius error
// (the reference uses at::allclose with 1e-3, :155); with EIR_DRIVER_DUMP=<dir>
// the inputs and the result are also written for the CPU oracle.
#include <cuda_runtime.h>
#include <chrono>
#include <cstdio>
#include <map>
#include <string>
#include <vector>
#include "BinaryContractionCuda.h"
#include "EinsumExpression.h"
#include "MemoryManager.h"
#include "driver_util.h"
#include "eir_cuda.h"

using einsum_ir::backend::BinaryContractionCuda;
using einsum_ir::frontend::EinsumExpressionAscii;
using namespace eir_driver;

namespace {

void usage() {
  std::fprintf(stderr,
               "Usage:\n"
               "  bench_binary einsum_string dimension_sizes dtype loop_order\n\n"
               "Arguments:\n"
               "  * einsum_string:    Einsum string with a binary contraction\n"
               "  * dimension_sizes:  Dimension sizes have to be in ascending order of the dimension ids.\n"
               "  * dtype:            FP32, FP64, BF16 or TF32, default: FP32.\n"
               "  * loop_order:       Loop execution strategy (accepted, not used by the GPU backend)\n\n"
               "Example:\n"
               "  ./bench_binary \"akmj,njk->anm\" \"16,64,32,512,512\" BF16\n");
}

// ZERO / MADD / no last touch contraction of the given dtype setup on `st`
struct Contraction {
  BinaryContractionCuda bc;
  einsum_ir::backend::MemoryManager mem;
  einsum_ir::err_t setup(std::map<int64_t, int64_t> const &sizes, std::vector<int64_t> const &l,
                         std::vector<int64_t> const &r, std::vector<int64_t> const &o,
                         einsum_ir::data_t dt_in, einsum_ir::data_t dt_out, int32_t comp,
                         cudaStream_t st) {
    bc.init((int64_t)l.size(), (int64_t)r.size(), (int64_t)o.size(), &sizes, &sizes, &sizes, nullptr,
            &sizes, nullptr, l.data(), r.data(), o.data(), nullptr, nullptr, &mem, dt_in, dt_in, dt_out,
            dt_out, einsum_ir::ZERO, einsum_ir::MADD, einsum_ir::UNDEFINED_KTYPE, 1);
    bc.set_compute_type(comp);
    bc.set_stream(st);
    return bc.compile();
  }
};

}  // namespace

int main(int argc, char *argv[]) {
  std::printf("running bench_binary!\n");
  if (argc < 3) {
    usage();
    return EXIT_FAILURE;
  }
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
  if (tensors.size() != 3) {
    std::fprintf(stderr, "Einsum string is not a binary contraction\n");
    return EXIT_FAILURE;
  }
  std::printf("parsed tensors:\n");
  for (auto const &t : tensors) std::printf("  %s\n", t.c_str());
  std::map<std::string, int64_t> name_to_id;
  EinsumExpressionAscii::parse_dim_ids(expr_std, name_to_id);
  std::printf("parsed dimension ids:\n");
  for (auto const &kv : name_to_id) std::printf("  %s: %lld\n", kv.first.c_str(), (long long)kv.second);
  std::string sizes_arg(argv[2]);
  std::vector<int64_t> size_vec;
  EinsumExpressionAscii::parse_dim_sizes(sizes_arg, size_vec);
  if (size_vec.size() != name_to_id.size()) {
    std::fprintf(stderr, "error: %zu dimension sizes for %zu dimensions\n", size_vec.size(),
                 name_to_id.size());
    return EXIT_FAILURE;
  }
  std::printf("parsed dimension sizes:\n");
  std::map<int64_t, int64_t> sizes;
  for (auto const &kv : name_to_id) {
    std::printf("  %s: %lld\n", kv.first.c_str(), (long long)size_vec[kv.second]);
    sizes[kv.second] = size_vec[kv.second];
  }
  std::string dtype = argc > 3 ? std::string(argv[3]) : std::string("FP32");
  if (dtype != "FP32" && dtype != "FP64" && dtype != "BF16" && dtype != "TF32") {
    std::fprintf(stderr, "failed to determine dtype\n");
    return EXIT_FAILURE;
  }
  std::printf("dtype: %s\n", dtype.c_str());
  if (argc > 4) std::printf("loop order: %s (not used by the GPU backend)\n", argv[4]);

  std::vector<int64_t> ids[3];
  std::vector<int64_t> shape[3];
  for (int t = 0; t < 3; ++t) {
    std::vector<std::string> names;
    EinsumExpressionAscii::split_string(tensors[t], ",", names);
    for (auto const &n : names) {
      ids[t].push_back(name_to_id[n]);
      shape[t].push_back(sizes[name_to_id[n]]);
    }
  }
  int64_t flops = 2;
  for (auto const &kv : sizes) flops *= kv.second;

  const int in_esize = dtype == "FP64" ? 8 : (dtype == "BF16" ? 2 : 4);
  const int out_esize = dtype == "FP64" ? 8 : 4;
  int64_t n[3];
  for (int t = 0; t < 3; ++t) {
    n[t] = 1;
    for (auto s : shape[t]) n[t] *= s;
  }
  DeviceTensor dl, dr, dout;
  std::vector<double> hl = upload(uniform(n[0], 1, 0.0, 1.0), in_esize, dl);
  std::vector<double> hr = upload(std::vector<double>((size_t)n[1], 1.0), in_esize, dr);
  upload(std::vector<double>((size_t)n[2], 0.0), out_esize, dout);
  cudaStream_t st;
  check_cuda(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate");

  std::printf("einsum_ir (B200):\n");
  const einsum_ir::data_t dt_in = dtype == "FP64" ? einsum_ir::FP64
                                : dtype == "BF16" ? einsum_ir::BF16 : einsum_ir::FP32;
  const einsum_ir::data_t dt_out = dtype == "FP64" ? einsum_ir::FP64 : einsum_ir::FP32;
  Contraction c;
  auto tp0 = std::chrono::steady_clock::now();
  einsum_ir::err_t err = c.setup(sizes, ids[0], ids[1], ids[2], dt_in, dt_out,
                                 dtype == "TF32" ? EIR_COMPUTE_TF32 : EIR_COMPUTE_DEFAULT, st);
  auto tp1 = std::chrono::steady_clock::now();
  if (err != einsum_ir::SUCCESS) {
    std::fprintf(stderr, "error: compile failed (%d): %s\n", (int)err, eir_last_error_string());
    return EXIT_FAILURE;
  }
  const double t_compile = std::chrono::duration<double>(tp1 - tp0).count();
  std::printf("  plan: %s\n", eir_plan_describe(c.bc.m_plan));
  const double t = time_calls([&] { c.bc.contract(dl.ptr, dr.ptr, dout.ptr); }, st);
  check_cuda(cudaStreamSynchronize(st), "contract");
  if (c.bc.m_last_status != EIR_SUCCESS || eir_check_device_errors(st) != EIR_SUCCESS) {
    std::fprintf(stderr, "error: contract failed: %s\n", eir_last_error_string());
    return EXIT_FAILURE;
  }
  std::printf("  time (compile): %g\n", t_compile);
  std::printf("  time (contract): %g\n", t);
  std::printf("  gflops: %g\n", 1e-9 * (double)flops / t);
  int64_t cmnk[4] = {1, 1, 1, 1};
  for (auto x : c.bc.m_sizes_c) cmnk[0] *= x;
  for (auto x : c.bc.m_sizes_m) cmnk[1] *= x;
  for (auto x : c.bc.m_sizes_n) cmnk[2] *= x;
  for (auto x : c.bc.m_sizes_k) cmnk[3] *= x;
  std::printf("  C M N K: %lld %lld %lld %lld\n", (long long)cmnk[0], (long long)cmnk[1],
              (long long)cmnk[2], (long long)cmnk[3]);
  std::printf("CSV_DATA: einsum_ir_b200,\"%s\",\"%s\",%s,%lld,%g,%g,%g\n", expr_arg.c_str(),
              sizes_arg.c_str(), dtype.c_str(), (long long)flops, t_compile, t, 1e-9 * (double)flops / t);

  // check against the FP64 CUDA-core contraction of the same values
  std::vector<double> got = download(dout);
  {
    Dump dump;  // EIR_DRIVER_DUMP: inputs and result for the CPU oracle
    dump.line("expr", expr_arg);
    dump.line("sizes", sizes_arg);
    dump.line("dtype", dtype);
    dump.tensor("in0", ids[0], shape[0], hl);
    dump.tensor("in1", ids[1], shape[1], hr);
    dump.tensor("out", ids[2], shape[2], got);
  }
  DeviceTensor rl, rr, rout;
  upload(hl, 8, rl);
  upload(hr, 8, rr);
  upload(std::vector<double>((size_t)n[2], 0.0), 8, rout);
  std::vector<double> ref;
  {
    CudaCoreOnly guard;
    Contraction cr;
    if (cr.setup(sizes, ids[0], ids[1], ids[2], einsum_ir::FP64, einsum_ir::FP64, EIR_COMPUTE_DEFAULT,
                 st) != einsum_ir::SUCCESS) {
      std::fprintf(stderr, "error: FP64 check contraction failed: %s\n", eir_last_error_string());
      return EXIT_FAILURE;
    }
    cr.bc.contract(rl.ptr, rr.ptr, rout.ptr);
    check_cuda(cudaStreamSynchronize(st), "check contraction");
    ref = download(rout);
  }
  ErrorReport r = compare(ref, got);
  const double tol = dtype == "FP64" ? 1e-12 : (dtype == "TF32" ? 1e-2 : 1e-5);
  std::printf("  relative error vs FP64 CUDA-core solution: %g\n", r.rel);
  cudaStreamDestroy(st);
  if (r.rel > tol) {
    std::fprintf(stderr, "error: einsum_ir solution is not close to the FP64 solution!\n");
    return EXIT_FAILURE;
  }
  std::printf("  results are close\n");
  std::printf("finished running bench_binary!\n");
  return EXIT_SUCCESS;
}
