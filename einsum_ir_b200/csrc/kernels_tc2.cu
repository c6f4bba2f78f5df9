// tcgen05 strided binary contraction on CTA pairs (cta_group::2) for sm_100a.
//
// A cluster of two CTAs on two SMs computes one 256 (primitive M) x BN
// (primitive N) output tile with M = 256 tensor-core MMAs issued by the even
// ("leader") CTA: each CTA stages 128 rows of A and BN/2 rows of B per K block
// in its own shared memory, the tensor cores of the pair read both halves, and
// each CTA's TMEM receives its 128 output rows x BN columns. Per SM this loads
// 128 + BN/2 operand rows per 128 x BN outputs instead of 128 + BN, which is
// what bounds the one-CTA kernel when its operands stream from L2.
//
// Each CTA loads only its own halves (plain TMA tile loads, no multicast); the
// loads of both CTAs complete on the leader's `full` barrier, whose expected
// byte count the leader posts for the pair. The leader's MMA issuer releases a
// ring stage in both CTAs (one commit to each CTA's `empty` barrier) and
// publishes a finished accumulator to both epilogues the same way. Both
// epilogues drain their own TMEM and arrive on the leader's `tempty` barrier.
//
// Warp roles per CTA: warp 0 = TMA producer, warp 1 = MMA issuer (leader) and
// TMEM owner (both CTAs allocate with cta_group::2), warps 2..9 = epilogue, two
// per TMEM lane quadrant with half of the columns each (fused first / last
// touch as in the one-CTA kernel). FP32-exact mode (3xTF32): warps 2..5 =
// epilogue, warps 6..9 split each CTA's staged FP32 tiles into hi / lo TF32
// parts; the loads of a CTA then complete on its own barrier and the MMA
// issuer waits for the converter warps of both CTAs. TF32 plans read operand
// copies that the planner's copy kernels have already rounded to the nearest
// TF32 value. Every wait is bounded; a timeout raises the abort flag in both
// CTAs and records a device error.
#include <cuda.h>
#include "eir_common.cuh"
#include "eir_params.h"
#include "eir_kernels.h"
#include "eir_launch.h"
#include "tc_tile.cuh"

namespace eir {

template <int KIND, int BN, int KSUB>
struct PairConfig {
  static constexpr int kEsize = (KIND == kKindBF16) ? 2 : 4;
  static constexpr int kBM = 128;                  // A rows (output rows) per CTA
  static constexpr int kBNh = BN / 2;              // B rows per CTA
  static constexpr int kBK = 128 / kEsize;         // K elements of one 128-byte swizzle row
  static constexpr int kMmaK = (KIND == kKindBF16) ? 16 : 8;
  static constexpr int kRowsPerBox = 128 / kEsize; // MN-major: rows per 128B box
  static constexpr int kASub = kBM * 128;
  static constexpr int kBSub = kBNh * 128;
  static constexpr int kABytes = KSUB * kASub;
  static constexpr int kBBytes = KSUB * kBSub;
  // FP32-exact mode keeps a hi and a lo TF32 copy of every staged operand
  static constexpr bool kSplit = (KIND == kKind3xTF32);
  static constexpr bool kConv = kSplit;                // converter warps (hi / lo split)
  static constexpr int kStageBytes = (kABytes + kBBytes) * (kSplit ? 2 : 1);
  static constexpr int kMaxStages = 8;
  static constexpr int kFit = (232448 - 1024 - 512) / kStageBytes;
  static constexpr int kStages = kFit < kMaxStages ? kFit : kMaxStages;
  // epilogue: 2 warps per TMEM lane quadrant (half the columns each), or 1
  // next to the 4 converter warps of the FP32-exact mode
  static constexpr int kEpiWarps = kConv ? 4 : 8;
  static constexpr int kConvWarps = kConv ? 4 : 0;
  static constexpr int kThreads = 32 * (2 + kEpiWarps + kConvWarps);
  static constexpr int kTmemCols = 2 * BN;         // double-buffered accumulator
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 512;
  static_assert(kStages >= 2, "at least two ring stages");
  static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM allocation must be a power of two");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kBNh % 16 == 0, "pair MMA N");
};

template <int KIND, int BN, int KSUB, bool A_MN, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairConfig<KIND, BN, KSUB>::kThreads, 1)
    tc_pair_contract_kernel(const __grid_constant__ CUtensorMap map_a,
                            const __grid_constant__ CUtensorMap map_b, const TcParams p,
                            const float *__restrict__ aux, float *__restrict__ out) {
  using Cfg = PairConfig<KIND, BN, KSUB>;
  constexpr int S = Cfg::kStages;
  constexpr int BK = Cfg::kBK;
  constexpr int BM = Cfg::kBM;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sA = smem;                   // S x kABytes
  uint8_t *sB = sA + S * Cfg::kABytes;  // S x kBBytes
  uint8_t *sAlo = sB + S * Cfg::kBBytes;                       // (split) S x kABytes
  uint8_t *sBlo = sAlo + (Cfg::kSplit ? S * Cfg::kABytes : 0);  // (split) S x kBBytes
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S * Cfg::kStageBytes);
  uint64_t *full = bars;                // S (leader's count both CTAs' bytes; converters: own bytes)
  uint64_t *empty = bars + S;           // S
  uint64_t *tfull = bars + 2 * S;       // 2
  uint64_t *tempty = bars + 2 * S + 2;  // 2 (leader's: epilogue warps of both CTAs)
  uint64_t *drain = bars + 2 * S + 4;   // 1 (leader: all MMAs done)
  uint64_t *conv = bars + 2 * S + 5;    // S (converters, leader's: converter warps of both CTAs)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * S + 5);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader
  const uint32_t peer = rank ^ 1u;
  const int64_t pair_id = blockIdx.x >> 1;
  const int64_t n_pairs = gridDim.x >> 1;
  const int n_kstages = (p.k_steps + KSUB - 1) / KSUB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * Cfg::kEpiWarps);
    }
    mbar_init(drain, 1);
    for (int s = 0; s < S; ++s) mbar_init(&conv[s], 2 * Cfg::kConvWarps);
    *abort_flag = 0;
    fence_barrier_init();
  }
  // the producer's first-tile set-up (kernel parameter loads, index
  // arithmetic) overlaps the rest of the prologue
  ProducerTile first_tile{};
  if (threadIdx.x == 0 && pair_id < p.total_tiles)
    first_tile = producer_tile<KSUB>(p, pair_id, n_kstages, 2 * BM, (int)rank * BM, BN,
                                     (int)rank * Cfg::kBNh);
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&map_a);
    tma_prefetch_map(&map_b);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();  // operands / output may come from the previous kernel of the stream
  const uint32_t peer_abort = mapa_shared(smem_u32((const void *)abort_flag), peer);
  auto raise_abort = [&](uint32_t code) {
    if (!*abort_flag) record_error(p.err, code);
    *abort_flag = 1;
    st_cluster_u32(peer_abort, 1u);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      const uint32_t full_leader = mapa_shared(smem_u32(full), 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int64_t t = pair_id; t < p.total_tiles && ok && !*abort_flag; t += n_pairs) {
        const ProducerTile pt = t == pair_id
                                    ? first_tile
                                    : producer_tile<KSUB>(p, t, n_kstages, 2 * BM, (int)rank * BM, BN,
                                                          (int)rank * Cfg::kBNh);
        // the TMA boxes of one K block of this CTA's operand halves
        auto k_block = [&](KWalk const &w, uint8_t *dA, uint8_t *dB, uint32_t bar) {
          const int a2 = slot_at(pt.sa, 0, w.ko0, w.ko1), a3 = slot_at(pt.sa, 1, w.ko0, w.ko1),
                    a4 = slot_at(pt.sa, 2, w.ko0, w.ko1);
          const int b2 = slot_at(pt.sb, 0, w.ko0, w.ko1), b3 = slot_at(pt.sb, 1, w.ko0, w.ko1),
                    b4 = slot_at(pt.sb, 2, w.ko0, w.ko1);
          const int kcol = w.kp * BK;
#pragma unroll
          for (int j = 0; j < (A_MN ? BM / Cfg::kRowsPerBox : 1); ++j) {
            const int x = A_MN ? pt.mrow + j * Cfg::kRowsPerBox : kcol, y = A_MN ? kcol : pt.mrow;
            tma_load_5d_pair(dA + j * BK * 128, &map_a, bar, x, y, a2, a3, a4);
          }
#pragma unroll
          for (int j = 0; j < (B_MN ? Cfg::kBNh / Cfg::kRowsPerBox : 1); ++j) {
            const int x = B_MN ? pt.nrow + j * Cfg::kRowsPerBox : kcol, y = B_MN ? kcol : pt.nrow;
            tma_load_5d_pair(dB + j * BK * 128, &map_b, bar, x, y, b2, b3, b4);
          }
        };
        KWalk kw = pt.kw;
        const int rot = pt.rot;
        for (int js = 0; js < n_kstages; ++js) {
          int ksg = js + rot;
          if (ksg >= n_kstages) ksg -= n_kstages;
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const int nsub = min(KSUB, p.k_steps - ksg * KSUB);
          // with converter warps each CTA's loads complete on its own barrier
          // (its converters wait there); otherwise on the leader's, for both
          if (Cfg::kConv) mbar_arrive_expect_tx(&full[stage], nsub * (Cfg::kASub + Cfg::kBSub));
          else if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * nsub * (Cfg::kASub + Cfg::kBSub));
          const uint32_t bar = Cfg::kConv ? smem_u32(&full[stage]) : full_leader + 8u * (uint32_t)stage;
          for (int sub = 0; sub < nsub; ++sub, kw.next(p))
            k_block(kw, sA + stage * Cfg::kABytes + sub * Cfg::kASub,
                    sB + stage * Cfg::kBBytes + sub * Cfg::kBSub, bar);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // wait until the MMAs released every stage, so that no commit of the
      // leader reaches this CTA's barriers after it exits
      for (int i = 0; i < S && ok && !*abort_flag; ++i) {
        if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) raise_abort(kErrTimeoutProducer);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc(KIND, 2 * BM, BN, A_MN, B_MN);
      constexpr bool kA32 = A_MN && Cfg::kEsize == 4, kB32 = B_MN && Cfg::kEsize == 4;
      constexpr uint32_t a_lay = kA32 ? kLayoutSw128Base32 : kLayoutSw128;
      constexpr uint32_t b_lay = kB32 ? kLayoutSw128Base32 : kLayoutSw128;
      constexpr uint32_t a_sbo = kA32 ? 512 : 1024, b_sbo = kB32 ? 512 : 1024;
      constexpr uint32_t a_lbo = A_MN ? BK * 128 : 16;
      constexpr uint32_t b_lbo = B_MN ? BK * 128 : 16;
      const uint32_t empty_peer = mapa_shared(smem_u32(empty), 1);
      const uint32_t tfull_peer = mapa_shared(smem_u32(tfull), 1);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const int kc = p.k_chunk > 0 ? p.k_chunk : n_kstages;  // stages per accumulation chunk
      for (int64_t t = pair_id; t < p.total_tiles && ok; t += n_pairs) {
        const int rot = k_rotation(t, n_kstages);
        for (int js0 = 0; js0 < n_kstages && ok; js0 += kc) {
        if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        const int js1 = min(js0 + kc, n_kstages);
        for (int js = js0; js < js1; ++js) {
          int ksg = js + rot;
          if (ksg >= n_kstages) ksg -= n_kstages;
          const int nsub = min(KSUB, p.k_steps - ksg * KSUB);
          if (!mbar_wait_bounded(Cfg::kConv ? &conv[stage] : &full[stage], phase, abort_flag)) {
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
                  umma_f16_pair(d_tmem, adesc, bdesc, idesc, accum);
                } else if (KIND == kKindTF32) {
                  umma_tf32_pair(d_tmem, adesc, bdesc, idesc, accum);
                } else {
                  const uint32_t alo_base = smem_u32(sAlo + stage * Cfg::kABytes + sub * Cfg::kASub);
                  const uint32_t blo_base = smem_u32(sBlo + stage * Cfg::kBBytes + sub * Cfg::kBSub);
                  const uint64_t alo = make_smem_desc(alo_base + a_off, a_lbo, a_sbo, a_lay);
                  const uint64_t blo = make_smem_desc(blo_base + b_off, b_lbo, b_sbo, b_lay);
                  umma_tf32_pair(d_tmem, alo, bdesc, idesc, accum);  // small terms first
                  umma_tf32_pair(d_tmem, adesc, blo, idesc, 1u);
                  umma_tf32_pair(d_tmem, adesc, bdesc, idesc, 1u);
                }
              }
            }
          }
          umma_commit_pair(smem_u32(&empty[stage]));
          umma_commit_pair(empty_peer + 8u * (uint32_t)stage);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&tfull[acc]));
        umma_commit_pair(tfull_peer + 8u * (uint32_t)acc);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
        }
      }
      // every MMA of this CTA pair has completed before TMEM is released
      umma_commit_pair(smem_u32(drain));
      if (!mbar_wait_bounded(drain, 0u, abort_flag) && !*abort_flag) ok = false;
      if (!ok) raise_abort(kErrTimeoutMma);
    }
  } else if (warp < 2 + Cfg::kEpiWarps) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = q * 32 + lane;
    constexpr int kCols = BN * 4 / Cfg::kEpiWarps;   // accumulator columns of this warp
    const int col0 = ((warp - 2) >> 2) * kCols;
    const uint32_t tempty_leader = mapa_shared(smem_u32(tempty), 0);
    const int fast = epilogue_kind(p);
    int acc = 0;
    uint32_t acc_phase = 0;
    const int kc = p.k_chunk > 0 ? p.k_chunk : n_kstages;
    const int n_chunks = (n_kstages + kc - 1) / kc;
    bool ok = true;
    for (int64_t t = pair_id; t < p.total_tiles && ok; t += n_pairs) {
      TileCoord c = decode_tile(p, t);
      for (int chunk = 0; chunk < n_chunks; ++chunk) {
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag)) {
        if (lane == 0) raise_abort(kErrTimeoutEpilogue);
        ok = false;
        break;
      }
      tc_fence_after();
      // -1: the whole K in one chunk; else first (0) / middle (1) / last (2)
      const int part = n_chunks == 1 ? -1 : (chunk == 0 ? 0 : (chunk + 1 == n_chunks ? 2 : 1));
      const int64_t m = c.mt * (2 * BM) + rank * BM + row;
      const bool mval = m < p.m_size;
      int64_t ob = m * p.so_m, ab = m * p.sa_m;
#pragma unroll
      for (int i = 0; i < kMaxTileLoops; ++i) {
        ob += c.l[i] * p.loop_so[i];
        ab += c.l[i] * p.loop_sa[i];
      }
      const int64_t n0 = c.nt * BN + col0;
      const int64_t so_n = p.so_n, sa_n = p.sa_n;
#pragma unroll 1
      for (int ch = 0; ch < kCols / 32; ++ch) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + col0 + ch * 32), v);
        tmem_ld_wait();
        if (!mval) continue;
        const int64_t nb = n0 + ch * 32;
        if (part < 0)
          store_chunk(p, v, out + ob + nb * so_n, aux + ab + nb * sa_n, nb, so_n, sa_n, fast);
        else
          store_chunk_part(p, v, out + ob + nb * so_n, aux + ab + nb * sa_n, nb, so_n, sa_n, part);
        if (p.peers.n > 0 && part != 0 && part != 1)  // final values only
          copy_to_peers(p, out + ob + nb * so_n, ob + nb * so_n, nb, so_n);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader + 8u * (uint32_t)acc);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else if constexpr (Cfg::kConv) {
    // ------------------------------------------------------------ converters (both CTAs)
    // each CTA splits its own staged halves, then every converter warp of
    // the pair arrives on the leader's conv barrier, which the MMA issuer
    // waits on
    const int ct = threadIdx.x - 32 * (2 + Cfg::kEpiWarps);  // 0 .. 32 * kConvWarps - 1
    constexpr int kCt = 32 * Cfg::kConvWarps;
    const uint32_t conv_leader = mapa_shared(smem_u32(conv), 0);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int64_t t = pair_id; t < p.total_tiles && ok; t += n_pairs) {
      for (int js = 0; js < n_kstages; ++js) {
        if (!mbar_wait_warp(&full[stage], phase, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t a = smem_u32(sA + stage * Cfg::kABytes);
        const uint32_t b = smem_u32(sB + stage * Cfg::kBBytes);
        split_stage<Cfg::kABytes, kCt>(a, smem_u32(sAlo + stage * Cfg::kABytes), ct);
        split_stage<Cfg::kBBytes, kCt>(b, smem_u32(sBlo + stage * Cfg::kBBytes), ct);
        fence_proxy_async_smem();  // the tensor cores read these tiles
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive_cluster(conv_leader + 8u * (uint32_t)stage);
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok && (threadIdx.x & 31) == 0) raise_abort(kErrTimeoutConvert);
  }

  // After an abort, copies or commits issued before it may still be landing in
  // this CTA's shared memory: give them time before the CTA can exit.
  if (threadIdx.x == 0 && *abort_flag) {
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // both CTAs done: no remote arrive or TMEM read is outstanding
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------- launchers
template <int KIND, int BN, int KSUB, bool A_MN, bool B_MN>
static cudaError_t launch_pair_t(CUtensorMap const &ma, CUtensorMap const &mb, TcParams const &p,
                                 float const *aux, float *out, cudaStream_t st) {
  using Cfg = PairConfig<KIND, BN, KSUB>;
  auto kern = tc_pair_contract_kernel<KIND, BN, KSUB, A_MN, B_MN>;
  static int max_clusters[32] = {0};  // per device: co-resident clusters of this instantiation
  int dev = 0;
  cudaGetDevice(&dev);
  int mc = dev < 32 ? max_clusters[dev] : 0;
  if (mc == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    e = cudaOccupancyMaxActiveClusters(&mc, kern, &cfg);
    if (e != cudaSuccess) return e;
    if (mc < 1) return cudaErrorInvalidConfiguration;
    if (dev < 32) max_clusters[dev] = mc;
  }
  int64_t pairs = p.total_tiles < mc ? p.total_tiles : mc;
  if (pairs < 1) return cudaSuccess;
  return launch_kernel(kern, dim3((unsigned)(2 * pairs)), dim3(Cfg::kThreads), Cfg::kSmemBytes, st,
                       ma, mb, p, aux, out);
}

template <int KIND, int BN, int KSUB>
static cudaError_t launch_pair_major(bool a_mn, bool b_mn, CUtensorMap const &ma,
                                     CUtensorMap const &mb, TcParams const &p, float const *aux,
                                     float *out, cudaStream_t st) {
  if (!a_mn && !b_mn) return launch_pair_t<KIND, BN, KSUB, false, false>(ma, mb, p, aux, out, st);
  if (!a_mn && b_mn) return launch_pair_t<KIND, BN, KSUB, false, true>(ma, mb, p, aux, out, st);
  if (a_mn && !b_mn) return launch_pair_t<KIND, BN, KSUB, true, false>(ma, mb, p, aux, out, st);
  return launch_pair_t<KIND, BN, KSUB, true, true>(ma, mb, p, aux, out, st);
}

cudaError_t launch_tc_pair_contract(int kind, int bn, int ksub, bool a_mn, bool b_mn,
                                    CUtensorMap const &ma, CUtensorMap const &mb, TcParams const &p,
                                    float const *aux, float *out, cudaStream_t st) {
  if (kind == kKindBF16 && bn == 256 && ksub == 1)
    return launch_pair_major<kKindBF16, 256, 1>(a_mn, b_mn, ma, mb, p, aux, out, st);
  if (kind == kKindBF16 && bn == 256 && ksub == 2)
    return launch_pair_major<kKindBF16, 256, 2>(a_mn, b_mn, ma, mb, p, aux, out, st);
  if (kind == kKindBF16 && bn == 128 && ksub == 2)
    return launch_pair_major<kKindBF16, 128, 2>(a_mn, b_mn, ma, mb, p, aux, out, st);
  if (kind == kKindBF16 && bn == 128 && ksub == 1)
    return launch_pair_major<kKindBF16, 128, 1>(a_mn, b_mn, ma, mb, p, aux, out, st);
  if (kind == kKindTF32 && bn == 256 && ksub == 1)
    return launch_pair_major<kKindTF32, 256, 1>(a_mn, b_mn, ma, mb, p, aux, out, st);
  if (kind == kKindTF32 && bn == 256 && ksub == 2)
    return launch_pair_major<kKindTF32, 256, 2>(a_mn, b_mn, ma, mb, p, aux, out, st);
  if (kind == kKindTF32 && bn == 128 && ksub == 2)
    return launch_pair_major<kKindTF32, 128, 2>(a_mn, b_mn, ma, mb, p, aux, out, st);
  if (kind == kKindTF32 && bn == 128 && ksub == 1)
    return launch_pair_major<kKindTF32, 128, 1>(a_mn, b_mn, ma, mb, p, aux, out, st);
  if (kind == kKind3xTF32 && bn == 256 && ksub == 1)
    return launch_pair_major<kKind3xTF32, 256, 1>(a_mn, b_mn, ma, mb, p, aux, out, st);
  if (kind == kKind3xTF32 && bn == 128 && ksub == 1)
    return launch_pair_major<kKind3xTF32, 128, 1>(a_mn, b_mn, ma, mb, p, aux, out, st);
  return cudaErrorInvalidValue;
}

}  // namespace eir
