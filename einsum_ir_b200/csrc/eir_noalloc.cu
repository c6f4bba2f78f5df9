// eir_contract_no_alloc: the binary contraction without any device allocation.
//
// Some callers cannot let a library call cudaMalloc: host frameworks that own
// all device memory through their own allocator (a caching allocator or an
// inference server's arena that reserves the GPU up front and forbids raw
// allocations afterwards), and latency-critical callers for which the device
// synchronisation and unpredictable cost of cudaMalloc/cudaFree on the hot path
// are not acceptable. eir_contract allocates its pre-permute workspace (and its
// device error word) lazily on first use; this entry point runs the same
// kernels but takes that scratch from a fixed array that is part of the
// library's device image.
//
// Limits and rules of use:
//  * the scratch is `g_static_scratch`, kStaticScratchBytes (8 MiB) per GPU.
//    Every GPU on which the library's kernels are loaded holds it until the
//    process exits. Its first 256 bytes are a header (the device error word of
//    the bounded waits); the rest holds the pre-permuted operand, so a plan
//    whose workspace exceeds kStaticOperandBytes is rejected with
//    EIR_INVALID_ARGUMENT and a message giving both sizes;
//  * the first call on a device does a one-time set-up with that device
//    current (the device address of the array is looked up with
//    cudaGetSymbolAddress, the SM count is read); make that first call before
//    any stream capture;
//  * all calls share the one array and it keeps the last call's contents: two
//    calls whose kernels overlap on the GPU (different streams, or host threads
//    racing on one device) race on the scratch. Serialise them, e.g. on one
//    stream. Nothing in the scratch needs to start at zero: the pre-permute
//    rewrites every byte the contraction reads, and the error word is zero
//    when the image is loaded and only ever set by a wait that gave up;
//  * a bounded device wait that gives up still ends the kernel; its code is
//    left in the header word and is not reported by this call.
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

extern "C" int eir_contract_no_alloc(eir_plan *p, void const *l, void const *r, void const *aux,
                                     void *out, void *stream) {
  if (p == nullptr || p->what != 1)
    return eir::api_set_error(EIR_INVALID_ARGUMENT, "not a contraction plan");
  if (p->empty) return EIR_SUCCESS;
  if (l == nullptr || r == nullptr || out == nullptr)
    return eir::api_set_error(EIR_NO_DATA_PTR_PROVIDED, "null operand pointer");
  bool uses_aux = p->first == EIR_KTYPE_COPY || p->first == EIR_KTYPE_ADD || p->last == EIR_KTYPE_ADD;
  if (uses_aux && aux == nullptr) return eir::api_set_error(EIR_NO_DATA_PTR_PROVIDED, "null aux pointer");
  if (p->cpx_inner != nullptr)
    return eir::api_set_error(EIR_INVALID_ARGUMENT,
                              "eir_contract_no_alloc: complex plans need their expansion workspace");
  if ((size_t)p->ws_bytes > kStaticOperandBytes) {
    char buf[192];
    std::snprintf(buf, sizeof(buf),
                  "eir_contract_no_alloc: plan needs %lld bytes of scratch, the static scratch "
                  "holds %lld bytes; use eir_contract",
                  (long long)p->ws_bytes, (long long)kStaticOperandBytes);
    return eir::api_set_error(EIR_INVALID_ARGUMENT, buf);
  }
  NoAllocDevice *d = nullptr;
  int rc = noalloc_device(&d);
  if (rc != EIR_SUCCESS) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  const bool aligned = !((reinterpret_cast<uintptr_t>(l) | reinterpret_cast<uintptr_t>(r)) & 15);
  if ((p->family != EIR_FAMILY_TC && p->family != EIR_FAMILY_DMMA) || !aligned) {
    cudaError_t e = eir::launch_simt_contract(p->dt_l, p->dt_r, p->dt_o, p->simt, l, r, aux, out, st);
    if (e != cudaSuccess) return eir::api_cuda_fail(e, "simt contraction launch");
    eir::api_count_launch();
    return EIR_SUCCESS;
  }

  void const *a_ptr = l, *b_ptr = r;
  if (p->prepack >= 0) {
    void *operand = d->scratch + kStaticHeaderBytes;
    eir::PermuteParams pp = p->pre->perm;
    void const *src = p->prepack == 0 ? l : r;
    if (pp.mode == 0 && pp.vec > 1 &&
        ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(operand)) %
         (pp.vec * p->pre->esize)))
      pp.vec = 1;
    cudaError_t e = eir::launch_permute(p->pre->esize, pp, src, operand, d->num_sms, st);
    if (e != cudaSuccess) return eir::api_cuda_fail(e, "permute launch");
    eir::api_count_launch();
    (p->prepack == 0 ? a_ptr : b_ptr) = operand;
  }

  CUtensorMap ma, mb;
  {
    std::lock_guard<std::mutex> lk(p->mu);
    if (p->cache_a.ptr != a_ptr) {
      rc = eir::api_encode_map(p->map_a, a_ptr, &p->cache_a.map);
      if (rc != EIR_SUCCESS) {
        p->cache_a.ptr = nullptr;
        return rc;
      }
      p->cache_a.ptr = a_ptr;
    }
    if (p->cache_b.ptr != b_ptr) {
      rc = eir::api_encode_map(p->map_b, b_ptr, &p->cache_b.map);
      if (rc != EIR_SUCCESS) {
        p->cache_b.ptr = nullptr;
        return rc;
      }
      p->cache_b.ptr = b_ptr;
    }
    ma = p->cache_a.map;
    mb = p->cache_b.map;
  }
  eir::TcParams tp = p->tcp;
  tp.err = reinterpret_cast<uint32_t *>(d->scratch);  // header word
  if (tp.split_k > 1) {  // split-K partial tiles after the pre-permuted operand, as in eir_contract
    float *ws = reinterpret_cast<float *>(d->scratch + kStaticHeaderBytes + p->split_ws_offset);
    return eir::api_launch_tc_split(p, ma, mb, tp, aux, out, ws, d->num_sms, st);
  }
  cudaError_t e = eir::api_launch_tc(p, ma, mb, tp, aux, out, d->num_sms, st);
  if (e != cudaSuccess) return eir::api_cuda_fail(e, "tc contraction launch");
  eir::api_count_launch();
  return EIR_SUCCESS;
}
