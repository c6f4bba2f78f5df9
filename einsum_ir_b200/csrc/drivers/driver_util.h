// Helpers shared by the command-line drivers (bench_expression, bench_binary):
// seeded host data, BF16 conversion, device buffers, CUDA-event timing loops
// and the relative-error report.
#ifndef EINSUM_IR_B200_DRIVER_UTIL_H
#define EINSUM_IR_B200_DRIVER_UTIL_H

#include <cuda_runtime.h>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <cstring>
#include <functional>
#include <random>
#include <string>
#include <vector>

namespace eir_driver {

inline void check_cuda(cudaError_t e, char const *what) {
  if (e != cudaSuccess) {
    std::fprintf(stderr, "error: %s: %s\n", what, cudaGetErrorString(e));
    std::exit(EXIT_FAILURE);
  }
}

// round-to-nearest-even FP32 -> BF16 bits (NaN kept quiet)
inline uint16_t to_bf16(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

inline float from_bf16(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float x;
  std::memcpy(&x, &u, 4);
  return x;
}

// i.i.d. values in [lo, hi) from a seeded generator (values held as double)
inline std::vector<double> uniform(int64_t n, uint64_t seed, double lo = -1.0, double hi = 1.0) {
  std::mt19937_64 g(seed);
  std::uniform_real_distribution<double> d(lo, hi);
  std::vector<double> v((size_t)n);
  for (auto &x : v) x = d(g);
  return v;
}

// storage types of the drivers: "FP32", "FP64", "BF16" (BF16 inputs, FP32 output)
struct DeviceTensor {
  void *ptr = nullptr;
  int64_t n = 0;
  int esize = 4;
  DeviceTensor() = default;
  DeviceTensor(DeviceTensor const &) = delete;
  DeviceTensor &operator=(DeviceTensor const &) = delete;
  ~DeviceTensor() {
    if (ptr) cudaFree(ptr);
  }
};

// copies `v` to the device in the storage type of `esize` (2 = BF16, 4 = FP32,
// 8 = FP64); returns the values the device holds (rounded) as doubles
inline std::vector<double> upload(std::vector<double> const &v, int esize, DeviceTensor &t) {
  t.n = (int64_t)v.size();
  t.esize = esize;
  check_cuda(cudaMalloc(&t.ptr, (size_t)(t.n > 0 ? t.n : 1) * esize), "cudaMalloc");
  std::vector<double> held(v.size());
  if (esize == 8) {
    check_cuda(cudaMemcpy(t.ptr, v.data(), v.size() * 8, cudaMemcpyHostToDevice), "cudaMemcpy");
    held = v;
  } else if (esize == 4) {
    std::vector<float> f(v.size());
    for (size_t i = 0; i < v.size(); ++i) {
      f[i] = (float)v[i];
      held[i] = f[i];
    }
    check_cuda(cudaMemcpy(t.ptr, f.data(), f.size() * 4, cudaMemcpyHostToDevice), "cudaMemcpy");
  } else {
    std::vector<uint16_t> b(v.size());
    for (size_t i = 0; i < v.size(); ++i) {
      b[i] = to_bf16((float)v[i]);
      held[i] = from_bf16(b[i]);
    }
    check_cuda(cudaMemcpy(t.ptr, b.data(), b.size() * 2, cudaMemcpyHostToDevice), "cudaMemcpy");
  }
  return held;
}

inline std::vector<double> download(DeviceTensor const &t) {
  std::vector<double> out((size_t)t.n);
  if (t.esize == 8) {
    check_cuda(cudaMemcpy(out.data(), t.ptr, out.size() * 8, cudaMemcpyDeviceToHost), "cudaMemcpy");
  } else {
    std::vector<float> f(out.size());
    check_cuda(cudaMemcpy(f.data(), t.ptr, f.size() * 4, cudaMemcpyDeviceToHost), "cudaMemcpy");
    for (size_t i = 0; i < f.size(); ++i) out[i] = f[i];
  }
  return out;
}

// Runs `fn` once to warm up, then enough repetitions for ~0.5 s (at least
// `min_reps`), timed with CUDA events on `st`. Returns seconds per call.
// Mean seconds per call of `fn` on `st`: one warm-up, one probe, then enough
// calls for about EIR_DRIVER_TIME_MS milliseconds (default 500), at least
// min_reps.
inline double time_calls(std::function<void()> const &fn, cudaStream_t st, int min_reps = 10) {
  double budget_ms = 500.0;
  if (char const *v = std::getenv("EIR_DRIVER_TIME_MS")) budget_ms = std::max(1.0, std::atof(v));
  fn();
  check_cuda(cudaStreamSynchronize(st), "warm-up");
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, st);
  fn();
  cudaEventRecord(e1, st);
  check_cuda(cudaEventSynchronize(e1), "probe run");
  float ms = 0;
  cudaEventElapsedTime(&ms, e0, e1);
  int64_t reps = (int64_t)(budget_ms / (ms > 1e-3 ? ms : 1e-3));
  if (reps < min_reps) reps = min_reps;
  if (reps > 100000) reps = 100000;
  cudaEventRecord(e0, st);
  for (int64_t r = 0; r < reps; ++r) fn();
  cudaEventRecord(e1, st);
  check_cuda(cudaEventSynchronize(e1), "timed runs");
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return ms * 1e-3 / (double)reps;
}

struct ErrorReport {
  double max_ref = 0, max_got = 0, max_diff = 0, frob_ref = 0, frob_got = 0, frob_diff = 0, rel = 0;
};

inline ErrorReport compare(std::vector<double> const &ref, std::vector<double> const &got) {
  ErrorReport r;
  for (size_t i = 0; i < ref.size(); ++i) {
    double d = got[i] - ref[i];
    r.max_ref = std::fmax(r.max_ref, std::fabs(ref[i]));
    r.max_got = std::fmax(r.max_got, std::fabs(got[i]));
    r.max_diff = std::fmax(r.max_diff, std::fabs(d));
    r.frob_ref += ref[i] * ref[i];
    r.frob_got += got[i] * got[i];
    r.frob_diff += d * d;
  }
  r.frob_ref = std::sqrt(r.frob_ref);
  r.frob_got = std::sqrt(r.frob_got);
  r.frob_diff = std::sqrt(r.frob_diff);
  r.rel = r.frob_ref > 0 ? r.frob_diff / r.frob_ref : r.frob_diff;
  return r;
}

inline void print_report(ErrorReport const &r, char const *ref_name) {
  std::printf("  maximum absolute entry in %s:  %g\n", ref_name, r.max_ref);
  std::printf("  maximum absolute entry in einsum_ir solution: %g\n", r.max_got);
  std::printf("  maximum element-wise difference:              %g\n", r.max_diff);
  std::printf("  frobenius norm of %s:          %g\n", ref_name, r.frob_ref);
  std::printf("  frobenius norm of einsum_ir solution:         %g\n", r.frob_got);
  std::printf("  frobenius norm of difference:                 %g\n", r.frob_diff);
  std::printf("  relative error:                               %g\n", r.rel);
}

// EIR_DRIVER_DUMP=<dir>: a driver writes the values its input tensors hold
// (<name>.f64, float64, the tensor's own layout), its result (out.f64) and a
// manifest (manifest.txt: one "key value..." line per fact: the command's
// arguments, each tensor's dimension ids and sizes, tree nodes), so that a
// test can recompute the result with the CPU oracle on the same values.
struct Dump {
  std::string dir;
  FILE *manifest = nullptr;
  Dump() {
    char const *v = std::getenv("EIR_DRIVER_DUMP");
    if (v == nullptr || *v == 0) return;
    dir = v;
    manifest = std::fopen((dir + "/manifest.txt").c_str(), "w");
    if (manifest == nullptr) {
      std::fprintf(stderr, "error: cannot write %s/manifest.txt\n", dir.c_str());
      std::exit(EXIT_FAILURE);
    }
  }
  ~Dump() {
    if (manifest) std::fclose(manifest);
  }
  bool on() const { return manifest != nullptr; }
  void line(std::string const &key, std::string const &value) {
    if (on()) std::fprintf(manifest, "%s %s\n", key.c_str(), value.c_str());
  }
  // "<name> ids i,j,... sizes a,b,..." and the values as <name>.f64
  void tensor(std::string const &name, std::vector<int64_t> const &ids, std::vector<int64_t> const &sizes,
              std::vector<double> const &values) {
    if (!on()) return;
    std::string s = "ids ";
    for (size_t i = 0; i < ids.size(); ++i) s += (i ? "," : "") + std::to_string(ids[i]);
    if (ids.empty()) s += "-";
    s += " sizes ";
    for (size_t i = 0; i < sizes.size(); ++i) s += (i ? "," : "") + std::to_string(sizes[i]);
    if (sizes.empty()) s += "-";
    line(name, s);
    FILE *f = std::fopen((dir + "/" + name + ".f64").c_str(), "wb");
    if (f == nullptr || std::fwrite(values.data(), sizeof(double), values.size(), f) != values.size()) {
      std::fprintf(stderr, "error: cannot write %s/%s.f64\n", dir.c_str(), name.c_str());
      std::exit(EXIT_FAILURE);
    }
    std::fclose(f);
  }
};

// Plans created while this guard lives run on the CUDA-core kernels only (the
// planner's tensor-core size threshold is raised out of reach): the drivers'
// FP64 reference solution.
struct CudaCoreOnly {
  std::string old;
  bool had = false;
  CudaCoreOnly() {
    char const *v = std::getenv("EIR_TC_MIN_OPS");
    had = v != nullptr;
    if (had) old = v;
    setenv("EIR_TC_MIN_OPS", "9223372036854775807", 1);
  }
  ~CudaCoreOnly() {
    if (had) setenv("EIR_TC_MIN_OPS", old.c_str(), 1);
    else unsetenv("EIR_TC_MIN_OPS");
  }
};

}  // namespace eir_driver

#endif
