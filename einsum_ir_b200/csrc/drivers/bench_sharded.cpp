// bench_sharded: BASELINE config 5 (zabcd,zcdef->zabef) with z split over the
// GPUs of a node, through the C++ ShardedContraction (one process per GPU).
// The reference has no multi-GPU driver; this one follows the report lines
// of its bench_expression (time / gflops of eval, CSV_DATA).
//
//   bench_sharded rank world exchange_dir [z size dtype]
//
// Every rank is started with the same arguments and its own rank (GPU rank %
// device count). The ranks exchange their CUDA IPC handles and synchronise
// through files in exchange_dir (a directory all ranks can see): the
// all-gather callback of eir_output_group_create can be any transport, and
// this one needs none beyond a shared file system. Defaults: z = 64, all other
// dims 48, FP64. Inputs: slab s of left and right holds seeded uniform
// [-1, 1) values that depend on s only, so every rank can rebuild any slab.
// Check: one slab of every rank's block, read from this rank's gathered full
// output, against the same slab contracted in FP64 on the CUDA-core kernels.
#include <cuda_runtime.h>
#include <sys/stat.h>
#include <unistd.h>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <string>
#include <thread>
#include <vector>
#include "BinaryContractionCuda.h"
#include "MemoryManager.h"
#include "ShardedContraction.h"
#include "driver_util.h"
#include "eir_cuda.h"

using einsum_ir::backend::ShardedContraction;
using namespace eir_driver;

namespace {

// all-gather through files: call k of rank r writes <dir>/k.r (complete
// before it becomes visible: written under another name, then renamed), then
// waits for the files of all ranks of call k (up to 120 s)
struct FileExchange {
  std::string dir;
  int32_t rank = 0, world = 1;
  int64_t calls = 0;
};

int file_allgather(void const *send, void *recv, int64_t bytes, void *user) {
  auto *x = static_cast<FileExchange *>(user);
  const int64_t k = x->calls++;
  const std::string mine = x->dir + "/" + std::to_string(k) + "." + std::to_string(x->rank);
  FILE *f = std::fopen((mine + ".tmp").c_str(), "wb");
  if (f == nullptr || std::fwrite(send, 1, (size_t)bytes, f) != (size_t)bytes) return 1;
  std::fclose(f);
  if (std::rename((mine + ".tmp").c_str(), mine.c_str()) != 0) return 1;
  auto t0 = std::chrono::steady_clock::now();
  for (int32_t r = 0; r < x->world; ++r) {
    const std::string p = x->dir + "/" + std::to_string(k) + "." + std::to_string(r);
    while (true) {
      FILE *g = std::fopen(p.c_str(), "rb");
      if (g != nullptr) {
        size_t n = std::fread(static_cast<char *>(recv) + r * bytes, 1, (size_t)bytes, g);
        std::fclose(g);
        if (n == (size_t)bytes) break;
      }
      if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(120)) return 1;
      std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
  }
  return 0;
}

int barrier(FileExchange &x) {
  std::vector<int32_t> all((size_t)x.world);
  int32_t one = 1;
  return file_allgather(&one, all.data(), sizeof(int32_t), &x);
}

// slab s of a [slab elements] tensor, seeded by (tensor, s)
std::vector<double> slab_values(int64_t n, int tensor, int64_t s) {
  return uniform(n, 1000003ull * (uint64_t)tensor + (uint64_t)s);
}

}  // namespace

int main(int argc, char *argv[]) {
  if (argc < 4) {
    std::fprintf(stderr,
                 "Usage:\n"
                 "  bench_sharded rank world exchange_dir [z size dtype]\n\n"
                 "Arguments:\n"
                 "  * rank, world:   this process's rank and the number of ranks (one GPU each)\n"
                 "  * exchange_dir:  a directory all ranks can read and write (handle exchange, barriers)\n"
                 "  * z, size, dtype: zabcd,zcdef->zabef sizes (default 64 48) and FP64 (default) or FP32\n");
    return EXIT_FAILURE;
  }
  // one hardware queue per stream (before the CUDA context exists): the copy
  // streams of eir_contract_gather wait on the kernel's slab counters, and a
  // blocked wait in a shared queue holds back the work behind it
  setenv("CUDA_DEVICE_MAX_CONNECTIONS", "32", 0);
  FileExchange x;
  x.rank = std::atoi(argv[1]);
  x.world = std::atoi(argv[2]);
  x.dir = argv[3];
  const int64_t z = argc > 4 ? std::atoll(argv[4]) : 64;
  const int64_t n = argc > 5 ? std::atoll(argv[5]) : 48;
  const std::string dtype = argc > 6 ? argv[6] : "FP64";
  if (x.world < 1 || x.rank < 0 || x.rank >= x.world || z % x.world != 0 || (dtype != "FP64" && dtype != "FP32")) {
    std::fprintf(stderr, "error: invalid arguments\n");
    return EXIT_FAILURE;
  }
  int devices = 0;
  check_cuda(cudaGetDeviceCount(&devices), "cudaGetDeviceCount");
  check_cuda(cudaSetDevice(x.rank % devices), "cudaSetDevice");
  const bool fp64 = dtype == "FP64";
  const int esize = fp64 ? 8 : 4;

  // dim ids: a 0, b 1, c 2, d 3, e 4, f 5, z 6 (sorted names)
  std::map<int64_t, int64_t> sizes;
  for (int64_t d = 0; d < 6; ++d) sizes[d] = n;
  sizes[6] = z;
  int64_t ids_l[5] = {6, 0, 1, 2, 3}, ids_r[5] = {6, 2, 3, 4, 5}, ids_o[5] = {6, 0, 1, 4, 5};
  ShardedContraction sc;
  sc.init(5, 5, 5, &sizes, ids_l, ids_r, ids_o, fp64 ? einsum_ir::FP64 : einsum_ir::FP32, 6, x.rank, x.world);
  cudaStream_t st;
  check_cuda(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate");
  sc.set_stream(st);
  if (sc.compile() != einsum_ir::SUCCESS) {
    std::fprintf(stderr, "error: compile failed: %s\n", eir_last_error_string());
    return EXIT_FAILURE;
  }
  const int64_t slab = n * n * n * n;  // elements of one z-slab of every tensor
  const int64_t zb = sc.block_size(), z0 = sc.block_begin();
  // this rank's input blocks (slab by slab from the seed) and the full output
  std::vector<double> hl, hr;
  for (int64_t s = z0; s < z0 + zb; ++s) {
    auto a = slab_values(slab, 0, s), b = slab_values(slab, 1, s);
    hl.insert(hl.end(), a.begin(), a.end());
    hr.insert(hr.end(), b.begin(), b.end());
  }
  DeviceTensor dl, dr, dout;
  upload(hl, esize, dl);
  upload(hr, esize, dr);
  upload(std::vector<double>((size_t)(z * slab), 0.0), esize, dout);
  if (sc.bind_output(dout.ptr, file_allgather, &x) != EIR_SUCCESS) {
    std::fprintf(stderr, "error: bind_output failed: %s\n", eir_last_error_string());
    return EXIT_FAILURE;
  }
  int rc = sc.contract(dl.ptr, dr.ptr, dout.ptr);  // warm-up
  check_cuda(cudaStreamSynchronize(st), "warm-up");
  if (rc != EIR_SUCCESS || barrier(x) != 0) {
    std::fprintf(stderr, "error: contract failed: %s\n", eir_last_error_string());
    return EXIT_FAILURE;
  }
  const double t_eval = time_calls([&] { rc |= sc.contract(dl.ptr, dr.ptr, dout.ptr); }, st, 3);
  check_cuda(cudaStreamSynchronize(st), "eval");
  if (rc != EIR_SUCCESS || eir_check_device_errors(st) != EIR_SUCCESS || barrier(x) != 0) {
    std::fprintf(stderr, "error: eval failed: %s\n", eir_last_error_string());
    return EXIT_FAILURE;
  }
  const int64_t flops = sc.num_ops();
  std::printf("rank %d of %d: z block [%lld, %lld)\n", x.rank, x.world, (long long)z0, (long long)(z0 + zb));
  std::printf("  #flops:         %lld\n", (long long)flops);
  std::printf("  time (eval):    %g\n", t_eval);
  std::printf("  gflops (eval):  %g\n", 1e-9 * (double)flops / t_eval);
  std::printf("CSV_DATA: einsum_ir_b200,bench_sharded,%d,%d,%lld,%lld,%s,%lld,%g,%g\n", x.rank, x.world,
              (long long)z, (long long)n, dtype.c_str(), (long long)flops, t_eval, 1e-9 * (double)flops / t_eval);

  // check: the first slab of every rank's block, as gathered into this rank's output
  std::map<int64_t, int64_t> ssz = sizes;
  ssz[6] = 1;
  double worst = 0.0;
  for (int32_t r = 0; r < x.world; ++r) {
    const int64_t s = (int64_t)r * zb;
    DeviceTensor cl, cr, co;
    upload(slab_values(slab, 0, s), 8, cl);
    upload(slab_values(slab, 1, s), 8, cr);
    upload(std::vector<double>((size_t)slab, 0.0), 8, co);
    {
      CudaCoreOnly guard;
      einsum_ir::backend::MemoryManager mem;
      einsum_ir::backend::BinaryContractionCuda bc;
      bc.init(5, 5, 5, &ssz, &ssz, &ssz, nullptr, &ssz, nullptr, ids_l, ids_r, ids_o, nullptr, nullptr, &mem,
              einsum_ir::FP64, einsum_ir::FP64, einsum_ir::FP64, einsum_ir::FP64, einsum_ir::ZERO, einsum_ir::MADD,
              einsum_ir::UNDEFINED_KTYPE, 1);
      bc.set_stream(st);
      if (bc.compile() != einsum_ir::SUCCESS) return EXIT_FAILURE;
      bc.contract(cl.ptr, cr.ptr, co.ptr);
      check_cuda(cudaStreamSynchronize(st), "check");
    }
    std::vector<double> ref = download(co);
    DeviceTensor view;  // the slab of the gathered output
    view.n = slab;
    view.esize = esize;
    view.ptr = static_cast<char *>(dout.ptr) + s * slab * esize;
    std::vector<double> got = download(view);
    view.ptr = nullptr;  // not owned
    worst = std::max(worst, compare(ref, got).rel);
  }
  std::printf("  relative error (first slab of every rank's block): %g\n", worst);
  barrier(x);  // no rank closes its mappings while another still copies
  sc.unbind();
  barrier(x);  // no rank frees its output while another still maps it
  cudaStreamDestroy(st);
  const double tol = fp64 ? 1e-12 : 1e-5;
  if (!(worst <= tol)) {
    std::fprintf(stderr, "error: relative error is large!\n");
    return EXIT_FAILURE;
  }
  return EXIT_SUCCESS;
}
