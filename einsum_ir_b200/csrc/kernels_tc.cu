// tcgen05 (5th-gen tensor core) strided binary contraction for sm_100a.
//
// One persistent CTA per SM walks output tiles of 128 (primitive M) x BN
// (primitive N). The remaining C / M / N dims are "tile loops" (scheduler
// coordinates); the K range is the primitive K dim (in blocks of one 128-byte
// swizzle row) times up to two outer K dims. Operands are read in their native
// strided layouts by 5-D TMA tensor maps (128B swizzle, K-major or MN-major
// per operand), staged in a shared-memory ring and consumed by tcgen05.mma
// issued from one thread, with the FP32 accumulator in TMEM (double buffered,
// so the epilogue of one tile overlaps the main loop of the next).
//
// A ring stage holds KSUB consecutive K blocks of both operands. The TMA
// producer / MMA consumer handshake costs a roughly fixed time per stage, so
// larger stages (KSUB = 2) raise the operand rate per SM. Tiles are walked in
// groups of `group_m` M tiles so CTAs running at the same time share operand
// tiles in L2.
//
// Warp roles: warp 0 = TMA producer, warp 1 = MMA issuer (+TMEM owner),
// warps 2..5 = epilogue (TMEM -> registers -> global, fused first/last touch:
// ZERO/COPY/ADD before, RELU/ADD after, aux read through broadcast strides),
// warps 6..9 (3xTF32 only) = converters (split_stage): store
// lo = x - trunc_TF32(x) of each staged FP32 tile next to it in shared memory
// (the staged x is the hi part, see tf32_lo_bits) so three MMAs (lo*hi + hi*lo
// + hi*hi) give an FP32-accurate product. TF32 plans read operand copies that
// the planner's copy kernels have already rounded to the nearest TF32 value.
//
// Semantics follow the reference loop engine: first touch at the first K
// step, last touch after the last (ContractionBackend.cpp:296-348,495-515;
// ContractionBackendTpp.cpp:15-62,80-163).
#include <cuda.h>
#include "eir_common.cuh"
#include "eir_params.h"
#include "eir_kernels.h"
#include "eir_launch.h"
#include "tc_tile.cuh"

namespace eir {

template <int KIND, int BN, int KSUB>
struct TcConfig {
  static constexpr int kEsize = (KIND == kKindBF16) ? 2 : 4;
  static constexpr int kBM = 128;
  static constexpr int kBK = 128 / kEsize;                 // K elements of one 128-byte swizzle row
  static constexpr int kMmaK = (KIND == kKindBF16) ? 16 : 8;
  static constexpr int kRowsPerBox = 128 / kEsize;         // MN-major: rows per 128B box
  static constexpr int kASub = kBM * 128;                  // A bytes of one K block
  static constexpr int kBSub = BN * 128;                   // B bytes of one K block
  static constexpr int kABytes = KSUB * kASub;             // per stage
  static constexpr int kBBytes = KSUB * kBSub;
  static constexpr bool kSplit = (KIND == kKind3xTF32);
  static constexpr bool kConv = kSplit;                    // converter warps 6..9
  static constexpr int kStageBytes = (kABytes + kBBytes) * (kSplit ? 2 : 1);
  static constexpr int kStages = 196608 / kStageBytes;
  static constexpr int kThreads = kConv ? 320 : 192;
  static constexpr int kTmemCols = 2 * BN;                 // double-buffered accumulator
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kBarBytes;
  static_assert(kStages >= 2, "at least two ring stages");
  static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM allocation must be a power of two");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

template <int KIND, int BN, int KSUB, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(TcConfig<KIND, BN, KSUB>::kThreads, 1)
    tc_contract_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b, const TcParams p,
                       const float *__restrict__ aux, float *__restrict__ out) {
  using Cfg = TcConfig<KIND, BN, KSUB>;
  constexpr int S = Cfg::kStages;
  constexpr int BK = Cfg::kBK;
  constexpr int BM = Cfg::kBM;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sA = smem;                                  // S x kABytes
  uint8_t *sB = sA + S * Cfg::kABytes;                 // S x kBBytes
  uint8_t *sAlo = sB + S * Cfg::kBBytes;               // (split) S x kABytes
  uint8_t *sBlo = sAlo + (Cfg::kSplit ? S * Cfg::kABytes : 0);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S * Cfg::kStageBytes);
  uint64_t *full = bars;                // S
  uint64_t *empty = bars + S;           // S
  uint64_t *conv = bars + 2 * S;        // S (converter warps only)
  uint64_t *tfull = bars + 3 * S;       // 2
  uint64_t *tempty = bars + 3 * S + 2;  // 2
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * S + 4);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // K walk in stages of KSUB K blocks
  const int n_kstages = (p.k_steps + KSUB - 1) / KSUB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 128);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  // the producer's first-tile set-up (kernel parameter loads, index
  // arithmetic) overlaps the rest of the prologue
  ProducerTile first_tile{};
  if (threadIdx.x == 0 && blockIdx.x < p.total_tiles)
    first_tile = producer_tile<KSUB>(p, blockIdx.x, n_kstages, BM, 0, BN, 0);
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&map_a);
    tma_prefetch_map(&map_b);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();  // operands / output may come from the previous kernel of the stream

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t t = blockIdx.x; t < p.total_tiles && !*abort_flag; t += gridDim.x) {
        const ProducerTile pt = t == (int64_t)blockIdx.x
                                    ? first_tile
                                    : producer_tile<KSUB>(p, t, n_kstages, BM, 0, BN, 0);
        // the TMA boxes of one K block into a ring stage
        auto k_block = [&](KWalk const &w, uint8_t *dA, uint8_t *dB, uint64_t *bar) {
          const int a2 = slot_at(pt.sa, 0, w.ko0, w.ko1), a3 = slot_at(pt.sa, 1, w.ko0, w.ko1),
                    a4 = slot_at(pt.sa, 2, w.ko0, w.ko1);
          const int b2 = slot_at(pt.sb, 0, w.ko0, w.ko1), b3 = slot_at(pt.sb, 1, w.ko0, w.ko1),
                    b4 = slot_at(pt.sb, 2, w.ko0, w.ko1);
          const int kcol = w.kp * BK;
#pragma unroll
          for (int j = 0; j < (A_MN ? BM / Cfg::kRowsPerBox : 1); ++j) {
            const int x = A_MN ? pt.mrow + j * Cfg::kRowsPerBox : kcol, y = A_MN ? kcol : pt.mrow;
            tma_load_5d(dA + j * BK * 128, &map_a, bar, x, y, a2, a3, a4);
          }
#pragma unroll
          for (int j = 0; j < (B_MN ? BN / Cfg::kRowsPerBox : 1); ++j) {
            const int x = B_MN ? pt.nrow + j * Cfg::kRowsPerBox : kcol, y = B_MN ? kcol : pt.nrow;
            tma_load_5d(dB + j * BK * 128, &map_b, bar, x, y, b2, b3, b4);
          }
        };
        KWalk kw = pt.kw;
        const int rot = pt.rot, kbeg = pt.kbeg, klen = pt.klen;
        for (int js = 0; js < klen; ++js) {
          int ksg = js + rot;
          if (ksg >= klen) ksg -= klen;
          if (rot > 0 && js == klen - rot) kw.seek(p, kbeg * KSUB);  // wrap to the item's first stage
          ksg += kbeg;
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag)) {
            if (!*abort_flag) record_error(p.err, kErrTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          const int nsub = min(KSUB, p.k_steps - ksg * KSUB);
          mbar_arrive_expect_tx(&full[stage], nsub * (Cfg::kASub + Cfg::kBSub));
          for (int sub = 0; sub < nsub; ++sub, kw.next(p))
            k_block(kw, sA + stage * Cfg::kABytes + sub * Cfg::kASub,
                    sB + stage * Cfg::kBBytes + sub * Cfg::kBSub, &full[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(KIND, BM, BN, A_MN, B_MN);
      // MN-major 32-bit operands use the 32-byte-atom swizzle (4-row K groups)
      constexpr bool kA32 = A_MN && Cfg::kEsize == 4, kB32 = B_MN && Cfg::kEsize == 4;
      constexpr uint32_t a_lay = kA32 ? kLayoutSw128Base32 : kLayoutSw128;
      constexpr uint32_t b_lay = kB32 ? kLayoutSw128Base32 : kLayoutSw128;
      constexpr uint32_t a_sbo = kA32 ? 512 : 1024, b_sbo = kB32 ? 512 : 1024;
      constexpr uint32_t a_lbo = A_MN ? BK * 128 : 16;
      constexpr uint32_t b_lbo = B_MN ? BK * 128 : 16;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const int kc = p.k_chunk > 0 ? p.k_chunk : n_kstages;  // stages per accumulation chunk
      for (int64_t t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
        const KRange kr = tile_krange(p, t, n_kstages);
        const int rot = k_rotation(t, kr.len);
        for (int js0 = 0; js0 < kr.len && ok; js0 += kc) {
        if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        const int js1 = min(js0 + kc, kr.len);
        for (int js = js0; js < js1; ++js) {
          int ksg = js + rot;
          if (ksg >= kr.len) ksg -= kr.len;
          ksg += kr.begin;
          const int nsub = min(KSUB, p.k_steps - ksg * KSUB);
          uint64_t *ready = Cfg::kConv ? &conv[stage] : &full[stage];
          if (!mbar_wait_bounded(ready, phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int sub = 0; sub < KSUB; ++sub) {
            if (sub < nsub) {
              const uint32_t a_base = smem_u32(sA + stage * Cfg::kABytes + sub * Cfg::kASub);
              const uint32_t b_base = smem_u32(sB + stage * Cfg::kBBytes + sub * Cfg::kBSub);
#pragma unroll
              for (int kk = 0; kk < BK / Cfg::kMmaK; ++kk) {
                const uint32_t a_off = A_MN ? kk * Cfg::kMmaK * 128 : kk * Cfg::kMmaK * Cfg::kEsize;
                const uint32_t b_off = B_MN ? kk * Cfg::kMmaK * 128 : kk * Cfg::kMmaK * Cfg::kEsize;
                const uint64_t adesc = make_smem_desc(a_base + a_off, a_lbo, a_sbo, a_lay);
                const uint64_t bdesc = make_smem_desc(b_base + b_off, b_lbo, b_sbo, b_lay);
                const uint32_t accum = (js > js0 || sub > 0 || kk > 0) ? 1u : 0u;
                if (KIND == kKindBF16) {
                  umma_f16(d_tmem, adesc, bdesc, idesc, accum);
                } else if (KIND == kKindTF32) {
                  umma_tf32(d_tmem, adesc, bdesc, idesc, accum);
                } else {
                  const uint32_t alo_base = smem_u32(sAlo + stage * Cfg::kABytes + sub * Cfg::kASub);
                  const uint32_t blo_base = smem_u32(sBlo + stage * Cfg::kBBytes + sub * Cfg::kBSub);
                  const uint64_t alo = make_smem_desc(alo_base + a_off, a_lbo, a_sbo, a_lay);
                  const uint64_t blo = make_smem_desc(blo_base + b_off, b_lbo, b_sbo, b_lay);
                  umma_tf32(d_tmem, alo, bdesc, idesc, accum);  // small terms first
                  umma_tf32(d_tmem, adesc, blo, idesc, 1u);
                  umma_tf32(d_tmem, adesc, bdesc, idesc, 1u);
                }
              }
            }
          }
          umma_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
        }
      }
      if (!ok) {
        if (!*abort_flag) record_error(p.err, kErrTimeoutMma);
        *abort_flag = 1;
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    const int kc = p.k_chunk > 0 ? p.k_chunk : n_kstages;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
      TileCoord c = decode_tile(p, t);
      const int n_chunks = (tile_krange(p, t, n_kstages).len + kc - 1) / kc;
      // split-K: this slice's partial tile goes to its workspace slice
      float *const tout =
          out + (p.split_k > 1 ? (int64_t)((uint32_t)t / (uint32_t)p.base_tiles) * p.ws_slice : 0);
      for (int chunk = 0; chunk < n_chunks; ++chunk) {
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag)) {
        if (!*abort_flag) record_error(p.err, kErrTimeoutEpilogue);
        *abort_flag = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      // -1: the whole K in one chunk; else first (0) / middle (1) / last (2)
      const int part = n_chunks == 1 ? -1 : (chunk == 0 ? 0 : (chunk + 1 == n_chunks ? 2 : 1));
      const int64_t m = c.mt * BM + row;
      const bool mval = m < p.m_size;
      int64_t ob = m * p.so_m, ab = m * p.sa_m;
#pragma unroll
      for (int i = 0; i < kMaxTileLoops; ++i) {
        ob += c.l[i] * p.loop_so[i];
        ab += c.l[i] * p.loop_sa[i];
      }
      const int64_t n0 = c.nt * BN;
      const int64_t so_n = p.so_n, sa_n = p.sa_n;
      const int fast = epilogue_kind(p);
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + ch * 32), v);
        tmem_ld_wait();
        if (!mval) continue;
        const int64_t nb = n0 + ch * 32;
        if (part < 0)
          store_chunk(p, v, tout + ob + nb * so_n, aux + ab + nb * sa_n, nb, so_n, sa_n, fast);
        else
          store_chunk_part(p, v, tout + ob + nb * so_n, aux + ab + nb * sa_n, nb, so_n, sa_n, part);
        if (p.peers.n > 0 && part != 0 && part != 1)  // final values only
          copy_to_peers(p, tout + ob + nb * so_n, ob + nb * so_n, nb, so_n);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else if constexpr (Cfg::kConv) {
    // ------------------------------------------------------------ converters
    const int ct = threadIdx.x - 192;  // 0..127
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
      const int klen = tile_krange(p, t, n_kstages).len;
      for (int js = 0; js < klen; ++js) {
        if (!mbar_wait_bounded(&full[stage], phase, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t a = smem_u32(sA + stage * Cfg::kABytes);
        const uint32_t b = smem_u32(sB + stage * Cfg::kBBytes);
        split_stage<Cfg::kABytes, 128>(a, smem_u32(sAlo + stage * Cfg::kABytes), ct);
        split_stage<Cfg::kBBytes, 128>(b, smem_u32(sBlo + stage * Cfg::kBBytes), ct);
        fence_proxy_async_smem();
        mbar_arrive(&conv[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok) {
      if (!*abort_flag) record_error(p.err, kErrTimeoutConvert);
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------- launchers
template <int KIND, int BN, int KSUB, bool A_MN, bool B_MN>
static cudaError_t launch_tc_t(CUtensorMap const &ma, CUtensorMap const &mb, TcParams const &p,
                               float const *aux, float *out, int num_sms, cudaStream_t st) {
  using Cfg = TcConfig<KIND, BN, KSUB>;
  auto kern = tc_contract_kernel<KIND, BN, KSUB, A_MN, B_MN>;
  static unsigned attr_set_mask = 0;  // one bit per device (attribute is per device)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 32 || !(attr_set_mask & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev < 32) attr_set_mask |= (1u << dev);
  }
  int64_t grid = p.total_tiles < num_sms ? p.total_tiles : num_sms;
  if (grid < 1) return cudaSuccess;
  return launch_kernel(kern, dim3((unsigned)grid), dim3(Cfg::kThreads), Cfg::kSmemBytes, st, ma, mb,
                       p, aux, out);
}

template <int KIND, int BN, int KSUB>
static cudaError_t launch_tc_major(bool a_mn, bool b_mn, CUtensorMap const &ma,
                                   CUtensorMap const &mb, TcParams const &p, float const *aux,
                                   float *out, int num_sms, cudaStream_t st) {
  if (!a_mn && !b_mn) return launch_tc_t<KIND, BN, KSUB, false, false>(ma, mb, p, aux, out, num_sms, st);
  if (!a_mn && b_mn) return launch_tc_t<KIND, BN, KSUB, false, true>(ma, mb, p, aux, out, num_sms, st);
  if (a_mn && !b_mn) return launch_tc_t<KIND, BN, KSUB, true, false>(ma, mb, p, aux, out, num_sms, st);
  return launch_tc_t<KIND, BN, KSUB, true, true>(ma, mb, p, aux, out, num_sms, st);
}

cudaError_t launch_tc_contract(int kind, int bn, int ksub, bool a_mn, bool b_mn,
                               CUtensorMap const &ma, CUtensorMap const &mb, TcParams const &p,
                               float const *aux, float *out, int num_sms, cudaStream_t st) {
  if (kind == kKindBF16 && bn == 256 && ksub == 1)
    return launch_tc_major<kKindBF16, 256, 1>(a_mn, b_mn, ma, mb, p, aux, out, num_sms, st);
  if (kind == kKindBF16 && bn == 256 && ksub == 2)
    return launch_tc_major<kKindBF16, 256, 2>(a_mn, b_mn, ma, mb, p, aux, out, num_sms, st);
  if (kind == kKindBF16 && bn == 128 && ksub == 1)
    return launch_tc_major<kKindBF16, 128, 1>(a_mn, b_mn, ma, mb, p, aux, out, num_sms, st);
  if (kind == kKindBF16 && bn == 128 && ksub == 2)
    return launch_tc_major<kKindBF16, 128, 2>(a_mn, b_mn, ma, mb, p, aux, out, num_sms, st);
  if (kind == kKindTF32 && bn == 256 && ksub == 1)
    return launch_tc_major<kKindTF32, 256, 1>(a_mn, b_mn, ma, mb, p, aux, out, num_sms, st);
  if (kind == kKindTF32 && bn == 256 && ksub == 2)
    return launch_tc_major<kKindTF32, 256, 2>(a_mn, b_mn, ma, mb, p, aux, out, num_sms, st);
  if (kind == kKindTF32 && bn == 128 && ksub == 1)
    return launch_tc_major<kKindTF32, 128, 1>(a_mn, b_mn, ma, mb, p, aux, out, num_sms, st);
  if (kind == kKindTF32 && bn == 128 && ksub == 2)
    return launch_tc_major<kKindTF32, 128, 2>(a_mn, b_mn, ma, mb, p, aux, out, num_sms, st);
  if (kind == kKind3xTF32 && bn == 128 && ksub == 1)
    return launch_tc_major<kKind3xTF32, 128, 1>(a_mn, b_mn, ma, mb, p, aux, out, num_sms, st);
  return cudaErrorInvalidValue;
}

int tc_block_k(int kind) { return kind == kKindBF16 ? 64 : (kind == 3 ? 16 : 32); }

// Split-K reduction: out = last_touch(first_touch(out, aux) + sum over s of
// ws[s]) for the dense workspace [slice][tile loops][n][m] of a split plan,
// summed in slice order (deterministic); peer copies as in the epilogues.
__global__ void __launch_bounds__(256)
    splitk_reduce_kernel(const TcParams p, const float *__restrict__ ws, const float *__restrict__ aux,
                         float *__restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t M = p.m_size, N = p.n_size, total = p.ws_slice;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = e % M, r = e / M;
    const int64_t n = r % N;
    int64_t l = r / N;
    int64_t o = m * p.so_m + n * p.so_n, a = m * p.sa_m + n * p.sa_n;
#pragma unroll
    for (int i = 0; i < kMaxTileLoops; ++i) {
      if (i < p.n_loops) {
        const int64_t li = l % p.loop_size[i];
        l /= p.loop_size[i];
        o += li * p.loop_so[i];
        a += li * p.loop_sa[i];
      }
    }
    float x = 0.0f;
    for (int s = 0; s < p.split_k; ++s) x += ws[(int64_t)s * total + e];
    if (p.first_touch == 3 /*COPY*/) x += aux[a];
    else if (p.first_touch == 2 /*ADD*/) x += out[o] + aux[a];
    else if (p.first_touch != 0 /*not ZERO*/) x += out[o];
    if (p.last_touch == 1 /*RELU*/) x = fmaxf(x, 0.0f);
    else if (p.last_touch == 2 /*ADD*/) x += aux[a];
    out[o] = x;
    for (int q = 0; q < p.peers.n; ++q) static_cast<float *>(p.peers.ptr[q])[o] = x;
  }
}

cudaError_t launch_splitk_reduce(TcParams const &p, float const *ws, float const *aux, float *out,
                                 int num_sms, cudaStream_t st) {
  int64_t blocks = (p.ws_slice + 255) / 256;
  const int64_t cap = (int64_t)num_sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return launch_kernel(splitk_reduce_kernel, dim3((unsigned)blocks), dim3(256), 0, st, p, ws, aux, out);
}

}  // namespace eir
