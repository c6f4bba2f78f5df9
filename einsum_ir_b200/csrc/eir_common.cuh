// Common device helpers for the einsum_ir B200 kernels (sm_100a only).
//
// Everything here is inline PTX for the Blackwell asynchronous machinery:
// mbarriers with bounded waits, TMA tensor loads (no multicast anywhere),
// tcgen05 TMEM allocation / MMA / commit / load.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace eir {

// TF32 compute: an FP32 value rounded to the nearest TF32 value, ties to even
// (10 explicit mantissa bits; the 13 low bits cleared). Infinities and NaNs
// stay as they are. The C oracle models TF32 with the same integer rounding,
// so the kernels and the oracle multiply identical operands.
__device__ __forceinline__ uint32_t round_tf32_bits(uint32_t u) {
  if ((u & 0x7f800000u) == 0x7f800000u) return u;
  u += 0x0fffu + ((u >> 13) & 1u);
  return u & 0xffffe000u;
}

// device-side error word codes (written with atomicCAS, first error wins)
enum : uint32_t {
  kErrNone = 0,
  kErrTimeoutProducer = 0x101,
  kErrTimeoutMma = 0x102,
  kErrTimeoutEpilogue = 0x103,
  kErrTimeoutConvert = 0x104,
};

// ~2 s at 1.9 GHz; a wait that needs longer than this means a broken pipeline
constexpr long long kWaitTimeoutCycles = 4000000000LL;

__device__ __forceinline__ uint32_t smem_u32(void const *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// 16-byte shared-memory accesses by shared-window address (LDS / STS even
// where the pointer was realigned through an integer cast and the compiler
// would otherwise emit generic accesses)
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Per-warpgroup register reallocation (all threads of the warpgroup execute
// it). An increase waits until other warpgroups have released enough of the
// registers the block was launched with, so a kernel's split must add up to at
// most its launch registers (threads x registers per thread).
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// Non-blocking test of an mbarrier phase.
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false if the wait gave up,
// either because `abort` was raised by another role of the CTA or because
// the cycle budget ran out (in which case the caller records an error).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  volatile int *abort) {
  if (mbar_try_wait(bar, parity)) return true;
  long long t0 = clock64();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitTimeoutCycles) return false;
  }
}

// Bounded wait for a whole warp that is not on the latency-critical path (the
// epilogue waiting for an accumulator, the TF32 splitter waiting for a stage):
// only lane 0 polls the barrier, with a short sleep between polls, while the
// other lanes wait at __syncwarp. Many threads polling an mbarrier in a tight
// loop slow down the TMA transactions that complete on the same barrier unit.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    if (!mbar_try_wait(bar, parity)) {
      long long t0 = clock64();
      while (true) {
        __nanosleep(128);
        if (mbar_try_wait(bar, parity)) break;
        if (*abort || clock64() - t0 > kWaitTimeoutCycles) {
          ok = 0;
          break;
        }
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  // every lane observes the completed phase itself (acquire); it is complete already
  if (ok) (void)mbar_try_wait(bar, parity);
  return ok != 0;
}

// ---- programmatic dependent launch ---------------------------------------
// A kernel launched with programmatic stream serialisation may start while
// the previous kernel of the stream is still running; pdl_wait() blocks until
// that kernel has completed and its memory is visible, so every thread calls
// it before its first global memory access. Kernels launched without the
// attribute return from it at once. pdl_launch_dependents() lets the next
// kernel of the stream start its prologue early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void record_error(uint32_t *err, uint32_t code) {
  if (err != nullptr) atomicCAS(err, 0u, code);
}

// ---- TMA ---------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_map(void const *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// 5-D tiled TMA load global -> shared, completion on an mbarrier (no multicast)
__device__ __forceinline__ void tma_load_5d(void *dst, void const *map, uint64_t *bar, int c0,
                                            int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// ---- tcgen05 -------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, one CTA, kind::f16 (bf16 inputs here)
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// arrive on `bar` once all previously issued tcgen05.mma of this thread completed
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM -> 32 registers per thread (row = lane)
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// tcgen05 shared-memory layout types (descriptor bits 61..63)
constexpr uint32_t kLayoutSw128 = 2;        // 128B swizzle, 16-byte atoms
constexpr uint32_t kLayoutSw128Base32 = 1;  // 128B swizzle, 32-byte atoms (32-bit MN-major)

// Shared-memory matrix descriptor for tcgen05 (sm_100 "version 1" format):
// start address, leading/stride byte offsets (16-byte units), layout type.
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo_bytes,
                                                   uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// ---- CTA pairs (clusters of two, tcgen05 cta_group::2) --------------------
// The even CTA of a pair is the leader: it issues the pair's MMAs. Shared
// addresses of the other CTA come from mapa (shared::cluster window).
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// address of the shared variable at `saddr` (this CTA) in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

// all threads of all CTAs of the cluster (a hardware barrier every thread reaches)
__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// arrive on an mbarrier given by its shared::cluster address (any CTA of the cluster)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
               : "memory");
}

__device__ __forceinline__ void st_cluster_u32(uint32_t addr_cluster, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr_cluster), "r"(v) : "memory");
}

// 5-D tiled TMA load into this CTA's shared memory whose completion is counted
// on an mbarrier of either CTA of the pair (the leader's); no multicast
__device__ __forceinline__ void tma_load_5d_pair(void *dst, void const *map, uint32_t bar_cluster,
                                                 int c0, int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// executed by the same warp of both CTAs of the pair; each CTA gets the address
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

// pair MMA (leader only): D (M = 256 over both CTAs' TMEM) (+)= A x B^T, where
// each CTA holds half of A's rows and half of B's rows at the same offsets
__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_tf32_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// arrive on the mbarrier at `bar_cluster` (this CTA's or the peer's) once all
// pair MMAs this thread issued so far have completed
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          bar_cluster)
      : "memory");
}

}  // namespace eir
