// FP64 strided binary contraction on the FP64 tensor cores (DMMA,
// mma.sync.m8n8k4.f64) for sm_100a.
//
// Same lowering as the tcgen05 kernel (TcParams, 5-D TMA tensor maps over the
// operands' native strides, tile loops and outer K loops, fused first/last
// touch), but tcgen05 has no FP64 kind, so the math runs on warp-level DMMA:
// warp 0 streams 128-row operand tiles with TMA (128B swizzle, K blocks of 16
// doubles) into a 4-stage ring; warps 1..8 each own a 64 x 32 slice of the
// 128 x 128 output tile, read A/B fragments from the swizzled stages
// (K-major or MN-major, by address arithmetic) and keep the accumulator in
// registers. Semantics: reference loop engine (ContractionBackend.cpp:296-348,
// 495-515; ContractionBackendTpp.cpp:80-163).
#include <cuda.h>
#include "eir_common.cuh"
#include "eir_params.h"
#include "eir_kernels.h"
#include "eir_launch.h"

namespace eir {

namespace {

constexpr int kDmmaBM = 128, kDmmaBN = 128, kDmmaBK = 16;  // 16 doubles = one 128-byte row
constexpr int kDmmaStages = 4;
constexpr int kDmmaTileBytes = 128 * 128;                   // one operand tile per stage
constexpr int kDmmaMathWarps = 16;  // 4 (M) x 4 (N) warps, 32 x 32 outputs each
constexpr int kDmmaThreads = 32 * (1 + kDmmaMathWarps);
constexpr int kDmmaSmem = 1024 + kDmmaStages * 2 * kDmmaTileBytes + 256;

// byte offset of element (row r, k) of a K-major 128B-swizzled tile [128 rows][16 doubles]
__device__ __forceinline__ uint32_t kmajor_off(int r, int k) {
  return (uint32_t)(r * 128 + ((((k >> 1) ^ (r & 7)) << 4) | ((k & 1) << 3)));
}
// byte offset of element (row r, k) of an MN-major tile: 8 boxes [16 k][16 rows]
__device__ __forceinline__ uint32_t mnmajor_off(int r, int k) {
  int b = r >> 4, rr = r & 15;
  return (uint32_t)(b * 2048 + k * 128 + ((((rr >> 1) ^ (k & 7)) << 4) | ((rr & 1) << 3)));
}

__device__ __forceinline__ void dmma(double &c0, double &c1, double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
               : "+d"(c0), "+d"(c1)
               : "d"(a), "d"(b));
}

struct DTile {
  int64_t mt, nt;
  int64_t l[kMaxTileLoops];
};

__device__ __forceinline__ DTile decode_dtile(TcParams const &p, int64_t t) {
  DTile c;
  const int64_t mn = (int64_t)p.m_tiles * p.n_tiles;
  int64_t u = t % mn;
  t /= mn;
  const int64_t gfull = (int64_t)p.group_m * p.n_tiles;
  const int64_t g = u / gfull;
  const int64_t first_m = g * p.group_m;
  const int64_t rem = p.m_tiles - first_m;
  const int64_t gm = rem < p.group_m ? rem : p.group_m;
  const int64_t r = u - g * gfull;
  c.mt = first_m + r % gm;
  c.nt = r / gm;
#pragma unroll
  for (int i = 0; i < kMaxTileLoops; ++i) {
    if (i < p.n_loops) {
      c.l[i] = t % p.loop_size[i];
      t /= p.loop_size[i];
    } else {
      c.l[i] = 0;
    }
  }
  return c;
}

__device__ __forceinline__ int dsrc(int8_t src, int64_t ko0, int64_t ko1, DTile const &c) {
  switch (src) {
    case kSrcKo0: return (int)ko0;
    case kSrcKo1: return (int)ko1;
    case kSrcLoop0: return (int)c.l[0];
    case kSrcLoop0 + 1: return (int)c.l[1];
    case kSrcLoop0 + 2: return (int)c.l[2];
    case kSrcLoop0 + 3: return (int)c.l[3];
    default: return 0;
  }
}

}  // namespace

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kDmmaThreads, 1)
    dmma_contract_kernel(const __grid_constant__ CUtensorMap map_a,
                         const __grid_constant__ CUtensorMap map_b, const TcParams p,
                         const double *__restrict__ aux, double *__restrict__ out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sA = smem;
  uint8_t *sB = smem + kDmmaStages * kDmmaTileBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + 2 * kDmmaStages * kDmmaTileBytes);
  uint64_t *full = bars;                 // kDmmaStages
  uint64_t *empty = bars + kDmmaStages;  // kDmmaStages (8 MMA warps arrive)
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

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_map(&map_a);
      tma_prefetch_map(&map_b);
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t t = blockIdx.x; t < p.total_tiles && !*abort_flag; t += gridDim.x) {
        DTile c = decode_dtile(p, t);
        const int mrow = (int)(c.mt * kDmmaBM), nrow = (int)(c.nt * kDmmaBN);
        for (int ks = 0; ks < k_steps; ++ks) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag)) {
            if (!*abort_flag) record_error(p.err, kErrTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          const int kp = ks % p.kp_blocks;
          const int64_t r = ks / p.kp_blocks;
          const int64_t ko0 = r % p.ko_size[0], ko1 = r / p.ko_size[0];
          mbar_arrive_expect_tx(&full[stage], 2 * kDmmaTileBytes);
          uint8_t *dA = sA + stage * kDmmaTileBytes, *dB = sB + stage * kDmmaTileBytes;
          const int kcol = kp * kDmmaBK;
          const int a2 = dsrc(p.a_src[2], ko0, ko1, c), a3 = dsrc(p.a_src[3], ko0, ko1, c),
                    a4 = dsrc(p.a_src[4], ko0, ko1, c);
          const int b2 = dsrc(p.b_src[2], ko0, ko1, c), b3 = dsrc(p.b_src[3], ko0, ko1, c),
                    b4 = dsrc(p.b_src[4], ko0, ko1, c);
          if (!A_MN) {
            tma_load_5d(dA, &map_a, &full[stage], kcol, mrow, a2, a3, a4);
          } else {
#pragma unroll
            for (int j = 0; j < kDmmaBM / 16; ++j)
              tma_load_5d(dA + j * 2048, &map_a, &full[stage], mrow + j * 16, kcol, a2, a3, a4);
          }
          if (!B_MN) {
            tma_load_5d(dB, &map_b, &full[stage], kcol, nrow, b2, b3, b4);
          } else {
#pragma unroll
            for (int j = 0; j < kDmmaBN / 16; ++j)
              tma_load_5d(dB + j * 2048, &map_b, &full[stage], nrow + j * 16, kcol, b2, b3, b4);
          }
          if (++stage == kDmmaStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else {
    // 16 math warps: 4 (M) x 4 (N), warp tile 32 x 32 = 4 x 4 DMMA tiles of 8 x 8
    constexpr int WI = 4, WJ = 4;
    const int mw = warp - 1;
    const int wm = (mw & 3) * 32, wn = (mw >> 2) * 32;
    const int g = lane >> 2, tq = lane & 3;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
      DTile c = decode_dtile(p, t);
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
#pragma unroll
        for (int kk = 0; kk < kDmmaBK; kk += 4) {
          double a[WI], b[WJ];
#pragma unroll
          for (int i = 0; i < WI; ++i) {
            const int r = wm + i * 8 + g, k = kk + tq;
            a[i] = *reinterpret_cast<const double *>(tA + (A_MN ? mnmajor_off(r, k) : kmajor_off(r, k)));
          }
#pragma unroll
          for (int j = 0; j < WJ; ++j) {
            const int r = wn + j * 8 + g, k = kk + tq;
            b[j] = *reinterpret_cast<const double *>(tB + (B_MN ? mnmajor_off(r, k) : kmajor_off(r, k)));
          }
#pragma unroll
          for (int i = 0; i < WI; ++i)
#pragma unroll
            for (int j = 0; j < WJ; ++j) dmma(acc[i][j][0], acc[i][j][1], a[i], b[j]);
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
      int64_t lo = 0, la = 0;
#pragma unroll
      for (int i = 0; i < kMaxTileLoops; ++i) {
        lo += c.l[i] * p.loop_so[i];
        la += c.l[i] * p.loop_sa[i];
      }
#pragma unroll
      for (int i = 0; i < WI; ++i) {
        const int64_t m = c.mt * kDmmaBM + wm + i * 8 + g;
        const bool mok = m < p.m_size;
#pragma unroll
        for (int j = 0; j < WJ; ++j) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int64_t n = c.nt * kDmmaBN + wn + j * 8 + 2 * tq + h;
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
            }
          }
        }
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
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kDmmaSmem);
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
