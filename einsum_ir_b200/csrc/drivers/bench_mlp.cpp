// bench_mlp: a multi-layer perceptron as a chain of EinsumNodes, the way the
// reference driver src/bench_mlp.cpp:82-330 builds one: every hidden layer is
// a binary-contraction node whose aux tensor is the layer's bias (outer size 1
// in the batch dim: broadcast), with a COPY first touch (out = bias), MADD and a
// RELU last touch; the last layer has no RELU. The weights are input nodes
// locked into internal memory with store_and_lock_data() before the timed
// evaluations (reference :305-311), as is the input with --lock-input.
//
//   bench_mlp [batch width layers dtype] [--data DIR] [--lock-input]
//
// Defaults: BASELINE config 3 (batch 8192, width 4096, 4 layers), FP32 data
// with FP32-accurate compute; dtype TF32 computes in TF32. Tensors: input
// X[b][f0], weight W_l[f_{l+1}][f_l] (the row-major layout of a torch Linear
// weight), bias B_l[f_{l+1}], output Y[b][f_L]. Data: --data DIR reads X.bin,
// W<l>.bin and B<l>.bin (raw little-endian float32, row-major) and writes the
// output to DIR/out.bin; without --data the values are seeded: X U[-1, 1),
// W N(0, 1/sqrt(width)), B U[-1, 1). Timing: eval() repeated for ~0.5 s with
// CUDA events; the report follows the reference (time / gflops of eval,
// num_ops).
#include <cuda_runtime.h>
#include <cstdio>
#include <cstring>
#include <map>
#include <random>
#include <string>
#include <vector>
#include "EinsumNode.h"
#include "MemoryManager.h"
#include "driver_util.h"
#include "eir_cuda.h"

using einsum_ir::backend::EinsumNode;
using namespace eir_driver;

namespace {

void usage() {
  std::fprintf(stderr,
               "Usage:\n"
               "  bench_mlp [batch width layers dtype] [--data DIR] [--lock-input]\n\n"
               "Arguments:\n"
               "  * batch, width, layers: default 8192 4096 4 (BASELINE config 3)\n"
               "  * dtype:       FP32 (FP32-accurate compute, default) or TF32\n"
               "  * --data DIR:  read X.bin, W<l>.bin, B<l>.bin (float32) from DIR, write DIR/out.bin\n"
               "  * --lock-input: also store_and_lock_data() the input before timing\n");
}

bool read_file(std::string const &path, std::vector<float> &v) {
  FILE *f = std::fopen(path.c_str(), "rb");
  if (f == nullptr) return false;
  size_t n = std::fread(v.data(), sizeof(float), v.size(), f);
  std::fclose(f);
  return n == v.size();
}

float *to_device(std::vector<float> const &v) {
  float *p = nullptr;
  check_cuda(cudaMalloc(&p, std::max<size_t>(v.size(), 1) * sizeof(float)), "cudaMalloc");
  check_cuda(cudaMemcpy(p, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice), "cudaMemcpy");
  return p;
}

}  // namespace

int main(int argc, char *argv[]) {
  std::vector<std::string> pos;
  std::string data_dir;
  bool lock_input = false;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    if (a == "--data" && i + 1 < argc) {
      data_dir = argv[++i];
    } else if (a == "--lock-input") {
      lock_input = true;
    } else if (a == "-h" || a == "--help") {
      usage();
      return EXIT_FAILURE;
    } else {
      pos.push_back(a);
    }
  }
  const int64_t batch = pos.size() > 0 ? std::atoll(pos[0].c_str()) : 8192;
  const int64_t width = pos.size() > 1 ? std::atoll(pos[1].c_str()) : 4096;
  const int64_t layers = pos.size() > 2 ? std::atoll(pos[2].c_str()) : 4;
  const std::string dtype = pos.size() > 3 ? pos[3] : "FP32";
  if (batch < 1 || width < 1 || layers < 1 || (dtype != "FP32" && dtype != "TF32")) {
    usage();
    return EXIT_FAILURE;
  }
  std::printf("running MLP using\n  batch: %lld\n  width: %lld\n  layers: %lld\n  dtype: %s\n"
              "  store and lock input: %d\n",
              (long long)batch, (long long)width, (long long)layers, dtype.c_str(), lock_input ? 1 : 0);

  // dim ids: 0 = batch, 1 + l = features entering layer l (1 + layers = output)
  std::map<int64_t, int64_t> sizes, sizes_aux;
  sizes[0] = batch;
  sizes_aux[0] = 1;  // the bias is broadcast over the batch
  for (int64_t l = 0; l <= layers; ++l) {
    sizes[1 + l] = width;
    sizes_aux[1 + l] = width;
  }

  // host data
  std::vector<float> x((size_t)(batch * width));
  std::vector<std::vector<float>> w((size_t)layers, std::vector<float>((size_t)(width * width)));
  std::vector<std::vector<float>> b((size_t)layers, std::vector<float>((size_t)width));
  if (!data_dir.empty()) {
    bool ok = read_file(data_dir + "/X.bin", x);
    for (int64_t l = 0; l < layers && ok; ++l)
      ok = read_file(data_dir + "/W" + std::to_string(l) + ".bin", w[l]) &&
           read_file(data_dir + "/B" + std::to_string(l) + ".bin", b[l]);
    if (!ok) {
      std::fprintf(stderr, "error: could not read the data files in %s\n", data_dir.c_str());
      return EXIT_FAILURE;
    }
  } else {
    std::mt19937_64 g(0);
    std::uniform_real_distribution<float> u(-1.0f, 1.0f);
    std::normal_distribution<float> nrm(0.0f, 1.0f / std::sqrt((float)width));
    for (auto &v : x) v = u(g);
    for (auto &wl : w)
      for (auto &v : wl) v = nrm(g);
    for (auto &bl : b)
      for (auto &v : bl) v = u(g);
  }
  float *d_x = to_device(x);
  std::vector<float *> d_w, d_b;
  for (int64_t l = 0; l < layers; ++l) {
    d_w.push_back(to_device(w[l]));
    d_b.push_back(to_device(b[l]));
  }
  float *d_out = nullptr;
  check_cuda(cudaMalloc(&d_out, (size_t)(batch * width) * sizeof(float)), "cudaMalloc");

  // the node chain: input, weights, hidden layers (the last one writes d_out)
  std::vector<std::vector<int64_t>> ids_w((size_t)layers), ids_h((size_t)layers);
  int64_t ids_x[2] = {0, 1};
  for (int64_t l = 0; l < layers; ++l) {
    ids_w[l] = {2 + l, 1 + l};
    ids_h[l] = {0, 2 + l};
  }
  einsum_ir::backend::MemoryManager memory;
  EinsumNode node_x;
  std::vector<EinsumNode> node_w((size_t)layers), node_h((size_t)layers);
  node_x.init(2, ids_x, &sizes, nullptr, einsum_ir::FP32, d_x, &memory);
  for (int64_t l = 0; l < layers; ++l)
    node_w[l].init(2, ids_w[l].data(), &sizes, nullptr, einsum_ir::FP32, d_w[l], &memory);
  for (int64_t l = 0; l < layers; ++l) {
    const bool last = l + 1 == layers;
    node_h[l].init(2, ids_h[l].data(), &sizes, &sizes_aux, nullptr, nullptr, nullptr, einsum_ir::FP32,
                   d_b[l], last ? d_out : nullptr, einsum_ir::COPY, einsum_ir::MADD,
                   last ? einsum_ir::UNDEFINED_KTYPE : einsum_ir::RELU,
                   l == 0 ? &node_x : &node_h[l - 1], &node_w[l], &memory, 1);
    node_h[l].m_compute = dtype == "TF32" ? EIR_COMPUTE_TF32 : EIR_COMPUTE_DEFAULT;
  }
  EinsumNode &root = node_h[layers - 1];
  cudaStream_t st = nullptr;
  check_cuda(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate");
  root.set_stream(st);

  auto t0 = std::chrono::steady_clock::now();
  einsum_ir::err_t err = root.compile();
  if (err != einsum_ir::SUCCESS) {
    std::fprintf(stderr, "error: failed to compile the MLP (err %d)\n", (int)err);
    return EXIT_FAILURE;
  }
  for (auto &n : node_w)
    if (n.store_and_lock_data() != einsum_ir::SUCCESS) {
      std::fprintf(stderr, "error: store_and_lock_data of a weight failed\n");
      return EXIT_FAILURE;
    }
  if (lock_input && node_x.store_and_lock_data() != einsum_ir::SUCCESS) {
    std::fprintf(stderr, "error: store_and_lock_data of the input failed\n");
    return EXIT_FAILURE;
  }
  check_cuda(cudaStreamSynchronize(st), "compile and lock");
  const double t_compile =
      std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();

  int status = EIR_SUCCESS;
  const double sec = time_calls([&] {
    int s = root.eval();
    if (status == EIR_SUCCESS) status = s;
  }, st, 3);
  if (status != EIR_SUCCESS || eir_check_device_errors(st) != EIR_SUCCESS) {
    std::fprintf(stderr, "error: evaluation failed: %s\n", eir_last_error_string());
    return EXIT_FAILURE;
  }
  const int64_t num_ops = root.num_ops();
  std::printf("time (compile + lock): %f\n", t_compile);
  std::printf("time (eval): %f\n", sec);
  std::printf("#flops: %lld\n", (long long)num_ops);
  std::printf("gflops (eval): %f\n", (double)num_ops / sec * 1e-9);
  std::printf("CSV_DATA: einsum_ir_b200,bench_mlp,%lld,%lld,%lld,%s,%lld,%f,%f\n", (long long)batch,
              (long long)width, (long long)layers, dtype.c_str(), (long long)num_ops, sec,
              (double)num_ops / sec * 1e-9);

  if (!data_dir.empty()) {
    std::vector<float> out((size_t)(batch * width));
    check_cuda(cudaMemcpy(out.data(), d_out, out.size() * sizeof(float), cudaMemcpyDeviceToHost), "cudaMemcpy");
    std::string p = data_dir + "/out.bin";
    FILE *f = std::fopen(p.c_str(), "wb");
    if (f == nullptr || std::fwrite(out.data(), sizeof(float), out.size(), f) != out.size()) {
      std::fprintf(stderr, "error: could not write %s\n", p.c_str());
      return EXIT_FAILURE;
    }
    std::fclose(f);
    std::printf("output written to %s\n", p.c_str());
  }
  for (auto &n : node_w) n.unlock_data();
  if (lock_input) node_x.unlock_data();
  cudaFree(d_x);
  for (auto *p : d_w) cudaFree(p);
  for (auto *p : d_b) cudaFree(p);
  cudaFree(d_out);
  cudaStreamDestroy(st);
  return EXIT_SUCCESS;
}
