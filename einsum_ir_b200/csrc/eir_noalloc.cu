// eir_contract_no_alloc: the binary contraction without any device allocation.
//
// Some callers cannot let a library call cudaMalloc: host frameworks that own
// all device memory through their own allocator (a caching allocator or an
// inference server's arena that reserves the GPU up front and forbids raw
// allocations afterwards), and latency-critical callers for which the device
// synchronisation and unpredictable cost of cudaMalloc/cudaFree on the hot path
// are not acceptable. eir_contract allocates its workspace (operand copies,
// split-K partial tiles) and its device error word lazily on first use; this
// entry point runs the same kernels but takes that scratch from a fixed array
// that is part of the library's device image.
//
// Limits and rules of use:
//  * the scratch is `g_static_scratch`, kStaticScratchBytes (8 MiB) per GPU.
//    Every GPU on which the library's kernels are loaded holds it until the
//    process exits. Its first 256 bytes are a header (the device error word of
//    the bounded waits); the rest holds the plan's workspace (re-laid-out or
//    TF32-rounded operand copies, split-K partial tiles), so a call whose
//    workspace exceeds kStaticOperandBytes is rejected with
//    EIR_INVALID_ARGUMENT and a message giving both sizes (a call that takes
//    the CUDA-core path, e.g. with unaligned operands, needs none);
//  * the first call on a device does a one-time set-up with that device
//    current (the device address of the array is looked up with
//    cudaGetSymbolAddress, the SM count is read); make that first call before
//    any stream capture;
//  * all calls share the one array and it keeps the last call's contents: two
//    calls whose kernels overlap on the GPU (different streams, or host threads
//    racing on one device) race on the scratch. Serialise them, e.g. on one
//    stream. Nothing in the scratch needs to start at zero: the operand copies
//    and the split-K slices write every byte that is read, and the error word is zero
//    when the image is loaded and only ever set by a wait that gave up;
//  * a bounded device wait that gives up still ends the kernel and leaves
//    its code in the header word; eir_check_device_errors (which allocates
//    nothing) reports and clears it, after which a later timeout is recorded
//    again (while the word is set, a further timeout is not recorded).
//
// The contraction itself is eir_contract's code path (eir::api_contract),
// given this scratch, the header word and the SM count instead of the
// plan's lazily allocated workspace and the device's error word.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdio>
#include <mutex>
#include <string>
#include "eir_kernels.h"
#include "eir_plan.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;  // 8 MiB
constexpr size_t kStaticHeaderBytes = 256;
constexpr size_t kStaticOperandBytes = kStaticScratchBytes - kStaticHeaderBytes;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

struct NoAllocDevice {
  bool ready = false;
  unsigned char *scratch = nullptr;  // device address of g_static_scratch
  int num_sms = 0;
};

std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[64];

// one-time per-device set-up, with that device current
int noalloc_device(NoAllocDevice **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return eir::api_cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return eir::api_set_error(EIR_CUDA_ERROR, "device index out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocDevice &d = g_noalloc_dev[dev];
  if (!d.ready) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return eir::api_cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return eir::api_cuda_fail(e, "cudaDeviceGetAttribute");
    d.scratch = static_cast<unsigned char *>(p);
    d.num_sms = n;
    d.ready = true;
  }
  *out = &d;
  return EIR_SUCCESS;
}

}  // namespace

namespace eir {
uint32_t *noalloc_error_word(int dev) {
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  return g_noalloc_dev[dev].ready ? reinterpret_cast<uint32_t *>(g_noalloc_dev[dev].scratch) : nullptr;
}
}  // namespace eir

extern "C" int eir_contract_no_alloc(eir_plan *p, void const *l, void const *r, void const *aux,
                                     void *out, void *stream) {
  if (p == nullptr || p->what != 1)
    return eir::api_set_error(EIR_INVALID_ARGUMENT, "not a contraction plan");
  if (p->empty) return EIR_SUCCESS;
  if (p->cpx_inner != nullptr)
    return eir::api_set_error(EIR_INVALID_ARGUMENT,
                              "eir_contract_no_alloc: complex plans need their expansion workspace");
  // the scratch this call uses: none when it takes the CUDA-core path
  const int64_t need = eir::api_workspace_needed(p, l, r);
  if ((size_t)need > kStaticOperandBytes) {
    char buf[192];
    std::snprintf(buf, sizeof(buf),
                  "eir_contract_no_alloc: plan needs %lld bytes of scratch, the static scratch "
                  "holds %lld bytes; use eir_contract",
                  (long long)need, (long long)kStaticOperandBytes);
    return eir::api_set_error(EIR_INVALID_ARGUMENT, buf);
  }
  NoAllocDevice *d = nullptr;
  int rc = noalloc_device(&d);
  if (rc != EIR_SUCCESS) return rc;
  return eir::api_contract(p, l, r, aux, out, nullptr, stream, nullptr, d->scratch + kStaticHeaderBytes,
                           reinterpret_cast<uint32_t *>(d->scratch), d->num_sms);
}
