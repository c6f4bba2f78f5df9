// FP64 strided binary contraction on the FP64 tensor cores (DMMA,
// mma.sync.m8n8k4.f64) for sm_100a.
//
// Same lowering as the tcgen05 kernel (TcParams, 5-D TMA tensor maps over the
// operands' native strides, tile loops and outer K loops, fused first/last
// touch), but tcgen05 has no FP64 kind, so the math runs on warp-level DMMA.
// Warp-specialised: warpgroup 0 gives its registers away (setmaxnreg) and one
// of its threads streams 128-row operand tiles with TMA (128B swizzle, K
// blocks of 16 doubles) into a 4-stage ring; warpgroups 1 and 2 (8 warps)
// each own a 32 x 64 slice of the 128 x 128 output tile, read A/B fragments
// from the swizzled stages (K-major or MN-major, by address arithmetic) and
// keep the accumulator in registers. Semantics: reference loop engine
// (ContractionBackend.cpp:296-348, 495-515; ContractionBackendTpp.cpp:80-163).
#include <cuda.h>
#include "eir_common.cuh"
#include "eir_params.h"
#include "eir_kernels.h"
#include "eir_launch.h"
#include "tc_tile.cuh"

namespace eir {

namespace {

constexpr int kDmmaBM = 128, kDmmaBN = 128, kDmmaBK = 16;  // 16 doubles = one 128-byte row
constexpr int kDmmaStages = 4;
constexpr int kDmmaTileBytes = 128 * 128;                   // one operand tile per stage
// 4 (M) x 2 (N) math warps, 32 x 64 outputs each (64 doubles of accumulator
// per thread). The register file is split over the 4 SM sub-partitions, so a
// launch's per-thread registers follow from its warps per sub-partition: 12
// warps (3 warpgroups) launch with 168; the producer warpgroup drops to 56 and
// the two math warpgroups rise to 224, which adds up to the launch's total
// (128 x 56 + 256 x 224 = 384 x 168). A 9-warp launch would cap the math at
// 168 registers and a 17-warp one at 96, both of which spill.
constexpr int kDmmaWarpsM = 4, kDmmaWarpsN = 2;
constexpr int kDmmaMathWarps = kDmmaWarpsM * kDmmaWarpsN;
constexpr int kDmmaThreads = 128 + 32 * kDmmaMathWarps;
constexpr int kDmmaLaunchRegs = 168, kDmmaProducerRegs = 56, kDmmaMathRegs = 224;
static_assert(kDmmaThreads == 384 && 65536 / kDmmaThreads / 8 * 8 == kDmmaLaunchRegs, "launch registers");
static_assert(128 * kDmmaProducerRegs + 32 * kDmmaMathWarps * kDmmaMathRegs <= kDmmaThreads * kDmmaLaunchRegs,
              "register split exceeds the launch's registers");
constexpr int kDmmaWI = kDmmaBM / kDmmaWarpsM / 8, kDmmaWJ = kDmmaBN / kDmmaWarpsN / 8;
constexpr int kDmmaSmem = 1024 + kDmmaStages * 2 * kDmmaTileBytes + 256;

__device__ __forceinline__ void dmma(double &c0, double &c1, double a, double b) {
  asm("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
               : "+d"(c0), "+d"(c1)
               : "d"(a), "d"(b));
}

}  // namespace

// Per-thread byte offsets of the DMMA fragments in one stage. The sum over the
// 16 k of a K block is order free, so MMA k-slot tq of K half h and pass q
// reads the physical k = 2 * pair(h, tq) + q, with pair(0, .) = {0, 2, 5, 7}
// and pair(1, .) = {1, 3, 4, 6} (A and B use the same map, so every product
// pairs equal k). A thread reads rows w + x * 8 + g (x = fragment index,
// g = lane / 4, tq = lane % 4); in the 128B swizzle its offsets are a thread
// constant plus an immediate per x:
//  K-major  [rows][16 doubles]: rows are 128 B and the 16-byte chunk index
//           (k / 2) ^ (row % 8) = pair ^ g does not depend on x, so
//           off = base[h] + x * 1024 and one 128-bit load fetches q = 0, 1;
//  MN-major 8 boxes [16 k][16 rows]: off = box * 2048 + k * 128 + chunk * 16
//           + (row % 2) * 8 with chunk = ((row % 16) / 2) ^ (k % 8); x moves
//           the box by x / 2 and flips chunk bit 2 (byte bit 6) by x % 2.
// The pair map keeps both forms free of shared-memory bank conflicts: in a
// K-major quarter warp (g = 0 / 1 on rows 128 B apart) the chunks pair ^ 0 and
// pair ^ 1 are disjoint, and in an MN-major half warp the four tq rows use
// k % 8 = 2 (pair % 4) + q, distinct in bits 1-2, so the 16 lanes cover 16
// different 8-byte bank pairs (k = 4 tq + 2 h + q collided tq = 0 with 2).
__device__ __forceinline__ int dmma_k_pair(int h, int tq) {
  return h == 0 ? (tq < 2 ? 2 * tq : 2 * tq + 1) : (tq < 2 ? 2 * tq + 1 : 2 * tq);
}

template <bool MN>
struct FragOffsets {
  uint32_t base[2][2];  // [h][q]; K-major uses base[h][0] only
  __device__ __forceinline__ FragOffsets(int w, int g, int tq) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int pair = dmma_k_pair(h, tq);
        const int k = 2 * pair + q;
        if (MN)
          base[h][q] = (uint32_t)((w >> 4) * 2048 + k * 128 + ((((g >> 1) ^ (k & 7))) << 4) + ((g & 1) << 3));
        else
          base[h][q] = (uint32_t)((w + g) * 128 + ((pair ^ g) << 4));
      }
  }
  // the pair (k, k + 1) of fragment x in K half h
  __device__ __forceinline__ double2 load(uint8_t const *tile, int h, int x) const {
    double2 v;
    if (MN) {
      const uint32_t flip = (uint32_t)(x & 1) << 6, box = (uint32_t)(x >> 1) * 2048;
      v.x = *reinterpret_cast<const double *>(tile + ((base[h][0] ^ flip) + box));
      v.y = *reinterpret_cast<const double *>(tile + ((base[h][1] ^ flip) + box));
    } else {
      v = *reinterpret_cast<const double2 *>(tile + base[h][0] + x * 1024);
    }
    return v;
  }
};

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kDmmaThreads, 1)
    dmma_contract_kernel(const __grid_constant__ CUtensorMap map_a,
                         const __grid_constant__ CUtensorMap map_b, const TcParams p,
                         const double *__restrict__ aux, double *__restrict__ out) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment by offsetting the shared array itself, so that the
  // compiler still knows the fragment loads are shared-memory loads
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t *sA = smem;
  uint8_t *sB = smem + kDmmaStages * kDmmaTileBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + 2 * kDmmaStages * kDmmaTileBytes);
  uint64_t *full = bars;                 // kDmmaStages
  uint64_t *empty = bars + kDmmaStages;  // kDmmaStages (the math warps arrive)
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 2 * kDmmaStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kDmmaStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDmmaMathWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();  // operands / output may come from the previous kernel of the stream
  const int k_steps = p.k_steps;

  if (warp < 4) {
    // ---- producer warpgroup: one thread issues every TMA load ----
    setmaxnreg_dec<kDmmaProducerRegs>();
    if (warp == 0 && lane == 0) {
      tma_prefetch_map(&map_a);
      tma_prefetch_map(&map_b);
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t t = blockIdx.x; t < p.total_tiles && !*abort_flag; t += gridDim.x) {
        // rotated, division-free K walk (the sum over K is order free)
        ProducerTile pt = producer_tile<1>(p, t, k_steps, kDmmaBM, 0, kDmmaBN, 0);
        for (int js = 0; js < k_steps; ++js) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag)) {
            if (!*abort_flag) record_error(p.err, kErrTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], 2 * kDmmaTileBytes);
          uint8_t *dA = sA + stage * kDmmaTileBytes, *dB = sB + stage * kDmmaTileBytes;
          const int kcol = pt.kw.kp * kDmmaBK, ko0 = pt.kw.ko0, ko1 = pt.kw.ko1;
          const int a2 = slot_at(pt.sa, 0, ko0, ko1), a3 = slot_at(pt.sa, 1, ko0, ko1),
                    a4 = slot_at(pt.sa, 2, ko0, ko1);
          const int b2 = slot_at(pt.sb, 0, ko0, ko1), b3 = slot_at(pt.sb, 1, ko0, ko1),
                    b4 = slot_at(pt.sb, 2, ko0, ko1);
          if (!A_MN) {
            tma_load_5d(dA, &map_a, &full[stage], kcol, pt.mrow, a2, a3, a4);
          } else {
#pragma unroll
            for (int j = 0; j < kDmmaBM / 16; ++j)
              tma_load_5d(dA + j * 2048, &map_a, &full[stage], pt.mrow + j * 16, kcol, a2, a3, a4);
          }
          if (!B_MN) {
            tma_load_5d(dB, &map_b, &full[stage], kcol, pt.nrow, b2, b3, b4);
          } else {
#pragma unroll
            for (int j = 0; j < kDmmaBN / 16; ++j)
              tma_load_5d(dB + j * 2048, &map_b, &full[stage], pt.nrow + j * 16, kcol, b2, b3, b4);
          }
          pt.kw.next(p);
          if (++stage == kDmmaStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else {
    // ---- math warpgroups ----
    setmaxnreg_inc<kDmmaMathRegs>();
    // warp tile (8 WI) x (8 WJ) = WI x WJ DMMA tiles of 8 x 8
    constexpr int WI = kDmmaWI, WJ = kDmmaWJ;
    const int mw = warp - 4;
    const int wm = (mw % kDmmaWarpsM) * (8 * WI), wn = (mw / kDmmaWarpsM) * (8 * WJ);
    const int g = lane >> 2, tq = lane & 3;
    const FragOffsets<A_MN> fa(wm, g, tq);
    const FragOffsets<B_MN> fb(wn, g, tq);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
      double acc[WI][WJ][2];
#pragma unroll
      for (int i = 0; i < WI; ++i)
#pragma unroll
        for (int j = 0; j < WJ; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;
      for (int ks = 0; ks < k_steps; ++ks) {
        if (!mbar_wait_bounded(&full[stage], phase, abort_flag)) {
          ok = false;
          break;
        }
        const uint8_t *tA = sA + stage * kDmmaTileBytes, *tB = sB + stage * kDmmaTileBytes;
        // The sum over the block's 16 k is order free: MMA k-slot tq takes the
        // physical k = 2 dmma_k_pair(h, tq) + q over the four MMAs (h, q), so a
        // thread's values for q = 0, 1 share one 16-byte chunk of a K-major tile.
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          double2 a[WI], b[WJ];
#pragma unroll
          for (int i = 0; i < WI; ++i) a[i] = fa.load(tA, h, i);
#pragma unroll
          for (int j = 0; j < WJ; ++j) b[j] = fb.load(tB, h, j);
          // two passes of WI * WJ independent DMMAs: an accumulator is revisited
          // only after all the others, which hides the DMMA latency
#pragma unroll
          for (int i = 0; i < WI; ++i)
#pragma unroll
            for (int j = 0; j < WJ; ++j) dmma(acc[i][j][0], acc[i][j][1], a[i].x, b[j].x);
#pragma unroll
          for (int i = 0; i < WI; ++i)
#pragma unroll
            for (int j = 0; j < WJ; ++j) dmma(acc[i][j][0], acc[i][j][1], a[i].y, b[j].y);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == kDmmaStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      // epilogue: fragment element (row g, cols 2tq, 2tq+1) of each 8 x 8 tile
      const TileCoord c = decode_tile(p, t);
      int64_t lo = 0, la = 0;
#pragma unroll
      for (int i = 0; i < kMaxTileLoops; ++i) {
        lo += (int64_t)c.l[i] * p.loop_so[i];
        la += (int64_t)c.l[i] * p.loop_sa[i];
      }
#pragma unroll
      for (int i = 0; i < WI; ++i) {
        const int64_t m = (int64_t)c.mt * kDmmaBM + wm + i * 8 + g;
        const bool mok = m < p.m_size;
#pragma unroll
        for (int j = 0; j < WJ; ++j) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int64_t n = (int64_t)c.nt * kDmmaBN + wn + j * 8 + 2 * tq + h;
            if (mok && n < p.n_size) {
              const int64_t o = lo + m * p.so_m + n * p.so_n;
              const int64_t a = la + m * p.sa_m + n * p.sa_n;
              double x = acc[i][j][h];
              if (p.first_touch == 3 /*COPY*/) x += aux[a];
              else if (p.first_touch == 2 /*ADD*/) x += out[o] + aux[a];
              else if (p.first_touch != 0 /*not ZERO*/) x += out[o];
              if (p.last_touch == 1 /*RELU*/) x = x > 0.0 ? x : 0.0;
              else if (p.last_touch == 2 /*ADD*/) x += aux[a];
              out[o] = x;
              for (int q = 0; q < p.peers.n; ++q) static_cast<double *>(p.peers.ptr[q])[o] = x;
            }
          }
        }
      }
      if (p.slab_ctr != nullptr) {
        // this warp's stores of tile t are visible device-wide before its
        // slab's count moves: a copy engine waiting on the count reads them
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(p.slab_ctr + slab_index(c, p.slab_loop), 1u);
      }
    }
    if (!ok && lane == 0) {
      if (!*abort_flag) record_error(p.err, kErrTimeoutMma);
      *abort_flag = 1;
    }
  }
  __syncthreads();
}

template <bool A_MN, bool B_MN>
static cudaError_t launch_dmma_t(CUtensorMap const &ma, CUtensorMap const &mb, TcParams const &p,
                                 double const *aux, double *out, int num_sms, cudaStream_t st) {
  auto kern = dmma_contract_kernel<A_MN, B_MN>;
  static unsigned attr_set_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 32 || !(attr_set_mask & (1u << dev))) {
    // the kernel's register split (setmaxnreg) is only sound for the launch
    // register count it was written for: with fewer, the math warpgroups'
    // increase could never be granted, so refuse to launch
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != kDmmaLaunchRegs) return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kDmmaSmem);
    if (e != cudaSuccess) return e;
    if (dev < 32) attr_set_mask |= (1u << dev);
  }
  int64_t grid = p.total_tiles < num_sms ? p.total_tiles : num_sms;
  if (grid < 1) return cudaSuccess;
  return launch_kernel(kern, dim3((unsigned)grid), dim3(kDmmaThreads), kDmmaSmem, st, ma, mb, p, aux,
                       out);
}

cudaError_t launch_dmma_contract(bool a_mn, bool b_mn, CUtensorMap const &ma, CUtensorMap const &mb,
                                 TcParams const &p, double const *aux, double *out, int num_sms,
                                 cudaStream_t st) {
  if (!a_mn && !b_mn) return launch_dmma_t<false, false>(ma, mb, p, aux, out, num_sms, st);
  if (!a_mn && b_mn) return launch_dmma_t<false, true>(ma, mb, p, aux, out, num_sms, st);
  if (a_mn && !b_mn) return launch_dmma_t<true, false>(ma, mb, p, aux, out, num_sms, st);
  return launch_dmma_t<true, true>(ma, mb, p, aux, out, num_sms, st);
}

}  // namespace eir
