// Tile scheduling and epilogue pieces shared by the tcgen05 contraction
// kernels (one CTA per tile in kernels_tc.cu, CTA pairs in kernels_tc2.cu).
#pragma once

#include <cstdint>
#include "eir_common.cuh"
#include "eir_params.h"

namespace eir {

enum { kKindBF16 = 0, kKindTF32 = 1, kKind3xTF32 = 2 };

// instruction descriptor for kind::f16 (bf16) / kind::tf32, FP32 accumulate
__host__ __device__ constexpr uint32_t make_idesc(int kind, int m, int n, bool a_mn, bool b_mn) {
  uint32_t fmt = (kind == kKindBF16) ? 1u : 2u;  // BF16 = 1, TF32 = 2
  return (1u << 4)                               // D format F32
         | (fmt << 7) | (fmt << 10)              // A / B format
         | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16)
         | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

struct TileCoord {
  int mt, nt;
  int l[kMaxTileLoops];
};

// tile index -> (M tile, N tile, tile-loop indices); M/N tiles in groups of
// group_m M tiles. 32-bit arithmetic: the planner keeps tile counts below 2^31.
__device__ __forceinline__ TileCoord decode_tile(TcParams const &p, int64_t tile) {
  TileCoord c;
  uint32_t t = (uint32_t)tile % (uint32_t)p.base_tiles;  // the output tile of a split-K slice
  const uint32_t mn = (uint32_t)p.m_tiles * (uint32_t)p.n_tiles;
  const uint32_t u = t % mn;
  t /= mn;
  const uint32_t gsz_full = (uint32_t)p.group_m * (uint32_t)p.n_tiles;
  const uint32_t g = u / gsz_full;
  const uint32_t first_m = g * (uint32_t)p.group_m;
  const uint32_t rem_m = (uint32_t)p.m_tiles - first_m;
  const uint32_t gm = rem_m < (uint32_t)p.group_m ? rem_m : (uint32_t)p.group_m;
  const uint32_t r = u - g * gsz_full;
  c.mt = (int)(first_m + r % gm);
  c.nt = (int)(r / gm);
#pragma unroll
  for (int i = 0; i < kMaxTileLoops; ++i) {
    if (i < p.n_loops) {
      c.l[i] = (int)(t % (uint32_t)p.loop_size[i]);
      t /= (uint32_t)p.loop_size[i];
    } else {
      c.l[i] = 0;
    }
  }
  return c;
}

// Tile-loop index of a tile coordinate for a run-time loop number (no
// dynamically indexed register array).
template <typename Coord>
__device__ __forceinline__ int slab_index(Coord const &c, int slab_loop) {
  int s = 0;
#pragma unroll
  for (int i = 0; i < kMaxTileLoops; ++i)
    if (i == slab_loop) s = c.l[i];
  return s;
}

__device__ __forceinline__ int src_coord(int8_t src, int ko0, int ko1, TileCoord const &c) {
  switch (src) {
    case kSrcKo0: return ko0;
    case kSrcKo1: return ko1;
    case kSrcLoop0: return c.l[0];
    case kSrcLoop0 + 1: return c.l[1];
    case kSrcLoop0 + 2: return c.l[2];
    case kSrcLoop0 + 3: return c.l[3];
    default: return 0;
  }
}

// TMA coordinates 2..4 of one operand for one tile: the tile-loop indices are
// fixed per tile, the outer K indices (ko0, ko1) change along the K walk.
struct SlotCoords {
  int base[3];
  int ko0_mask, ko1_mask;  // bit j: coordinate 2 + j is ko0 / ko1
};

__device__ __forceinline__ SlotCoords slot_coords(int8_t const (&src)[5], TileCoord const &c) {
  SlotCoords s;
  s.ko0_mask = s.ko1_mask = 0;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    s.base[j] = src_coord(src[2 + j], 0, 0, c);
    if (src[2 + j] == kSrcKo0) s.ko0_mask |= 1 << j;
    if (src[2 + j] == kSrcKo1) s.ko1_mask |= 1 << j;
  }
  return s;
}

__device__ __forceinline__ int slot_at(SlotCoords const &s, int j, int ko0, int ko1) {
  return s.base[j] + (((s.ko0_mask >> j) & 1) ? ko0 : 0) + (((s.ko1_mask >> j) & 1) ? ko1 : 0);
}

// Position (kp, ko0, ko1) of K block ks = kp + kp_blocks * (ko0 + ko_size0 * ko1),
// advanced without divisions: the producer thread issues every TMA load of
// the CTA, so its per-K-block instruction count bounds the operand rate.
struct KWalk {
  int ks, kp, ko0, ko1;
  __device__ __forceinline__ void seek(TcParams const &p, int k) {
    ks = k;
    kp = k % p.kp_blocks;
    const int r = k / p.kp_blocks;
    ko0 = r % (int)p.ko_size[0];
    ko1 = r / (int)p.ko_size[0];
  }
  // next K block; the walk wraps from the last block to block 0
  __device__ __forceinline__ void next(TcParams const &p) {
    if (++ks == p.k_steps) {
      ks = kp = ko0 = ko1 = 0;
    } else if (++kp == p.kp_blocks) {
      kp = 0;
      if (++ko0 == (int)p.ko_size[0]) {
        ko0 = 0;
        ++ko1;
      }
    }
  }
};

// K stages [begin, begin + len) of work item t (all of K without split-K)
struct KRange {
  int begin, len;
};
__device__ __forceinline__ KRange tile_krange(TcParams const &p, int64_t t, int n_kstages) {
  KRange r{0, n_kstages};
  if (p.split_k > 1) {
    const int s = (int)((uint32_t)t / (uint32_t)p.base_tiles);
    r.begin = (int)((int64_t)s * n_kstages / p.split_k);
    r.len = (int)((int64_t)(s + 1) * n_kstages / p.split_k) - r.begin;
  }
  return r;
}

// Start offset (in stages) of a tile's K walk. Tiles running at the same time
// start at different K positions so they do not all fetch the same operand
// lines at once (the sum over K is order independent up to FP32 rounding).
// Producer and MMA issuer only need to agree on the order of stages; the first
// MMA of a tile's walk always initialises the accumulator.
__device__ __forceinline__ int k_rotation(int64_t t, int n_stages) {
  if (n_stages <= 1) return 0;
  return (int)(((uint32_t)t * 7u) % (uint32_t)n_stages);
}

// Per-tile set-up of the TMA producer: tile coordinates, the operand row
// origins, the fixed TMA coordinates and the start of the rotated K walk.
struct ProducerTile {
  TileCoord c;
  int rot, mrow, nrow;
  int kbeg, klen;  // the work item's K stages (tile_krange)
  SlotCoords sa, sb;
  KWalk kw;
};

// m_rows / n_cols: output rows / columns of a tile; m_off / n_off: first row
// of this CTA's operand half within its tile (CTA pairs), else 0
template <int KSUB>
__device__ __forceinline__ ProducerTile producer_tile(TcParams const &p, int64_t t, int n_kstages,
                                                      int m_rows, int m_off, int n_cols, int n_off) {
  ProducerTile pt;
  pt.c = decode_tile(p, t);
  const KRange kr = tile_krange(p, t, n_kstages);
  pt.kbeg = kr.begin;
  pt.klen = kr.len;
  pt.rot = k_rotation(t, kr.len);
  pt.mrow = pt.c.mt * m_rows + m_off;
  pt.nrow = pt.c.nt * n_cols + n_off;
  pt.sa = slot_coords(p.a_src, pt.c);
  pt.sb = slot_coords(p.b_src, pt.c);
  pt.kw.seek(p, (kr.begin + pt.rot) * KSUB);
  return pt;
}

// FP32-exact mode (3xTF32): x = hi + lo with hi = x truncated to TF32 and
// lo = x - hi (exact in FP32); three TF32 MMAs lo*hi + hi*lo + hi*hi give an
// FP32-accurate product (the error-compensated TF32 method). The tensor core
// reads a TF32 operand from an FP32 word by ignoring its 13 low mantissa bits,
// so the staged x already is hi: only lo has to be computed and stored. The
// FP32 parity tests (relative error ~1e-6 against the oracle) pin this.
__device__ __forceinline__ uint32_t tf32_lo_bits(uint32_t u) {
  const float v = __uint_as_float(u);
  return __float_as_uint(v - __uint_as_float(u & 0xFFFFE000u));
}

// hi / lo split of one staged FP32 operand of BYTES at shared address `src`:
// lo(x) is stored at the same offset from `dst`. Thread `t` of NT handles
// 16-byte chunks t, t + NT, ... in batches of 8 independent loads, so the
// shared-memory latency overlaps instead of adding up per chunk.
template <int BYTES, int NT>
__device__ __forceinline__ void split_stage(uint32_t src, uint32_t dst, int t) {
  constexpr int kChunks = BYTES / 16 / NT;  // 16-byte chunks per thread
  static_assert(BYTES % (16 * NT) == 0, "whole chunks per thread");
  constexpr int kBatch = kChunks < 8 ? kChunks : 8;
  static_assert(kChunks % kBatch == 0, "whole batches");
#pragma unroll
  for (int b = 0; b < kChunks; b += kBatch) {
    uint4 v[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) v[j] = lds128(src + (uint32_t)(((b + j) * NT + t) * 16));
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      v[j].x = tf32_lo_bits(v[j].x);
      v[j].y = tf32_lo_bits(v[j].y);
      v[j].z = tf32_lo_bits(v[j].z);
      v[j].w = tf32_lo_bits(v[j].w);
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) sts128(dst + (uint32_t)(((b + j) * NT + t) * 16), v[j]);
  }
}

// Epilogue variant of a plan: 0 = ZERO first touch and no last touch, 1 = COPY
// (bias) first touch with no last touch or RELU, 2 = anything else.
__device__ __forceinline__ int epilogue_kind(TcParams const &p) {
  return (p.first_touch == 0 && p.last_touch == 99) ? 0
       : (p.first_touch == 3 && (p.last_touch == 99 || p.last_touch == 1)) ? 1 : 2;
}

// One accumulation chunk of a long K walk (TcParams::k_chunk), 32 columns of
// one output row. part 0: the first chunk, with the plan's first touch;
// part 1: a middle chunk, added to the partial sum stored by the previous
// chunk; part 2: the last chunk, added, then the last touch. The partial sums
// live in the output itself: the same thread wrote them, so they are visible.
// Every load is issued before the first store (the compiler cannot reorder
// them itself: the addresses may alias), so the 32 reads overlap.
__device__ __forceinline__ void store_chunk_part(TcParams const &p, uint32_t const (&v)[32], float *op,
                                                 const float *ap, int64_t nb, int64_t so_n, int64_t sa_n,
                                                 int part) {
  const int64_t rem = p.n_size - nb;
  const int lim = rem < 32 ? (int)rem : 32;
  // the partial sum (or, for the first chunk, what the first touch reads)
  const bool read_out = part != 0 || (p.first_touch != 0 && p.first_touch != 3);
  const bool read_aux = (part == 0 && (p.first_touch == 2 || p.first_touch == 3)) ||
                        (part == 2 && p.last_touch == 2);
  const bool add_aux_first = part == 0 && (p.first_touch == 2 || p.first_touch == 3);
  const bool relu = part == 2 && p.last_touch == 1;
  const bool add_aux_last = part == 2 && p.last_touch == 2;
  // two halves of 16 columns: 32 loads in flight, few registers
#pragma unroll
  for (int h = 0; h < 32; h += 16) {
    float prev[16], bias[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      prev[j] = (read_out && h + j < lim) ? op[(h + j) * so_n] : 0.0f;
      bias[j] = (read_aux && h + j < lim) ? ap[(h + j) * sa_n] : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (h + j < lim) {
        float x = __uint_as_float(v[h + j]) + prev[j];
        if (add_aux_first) x += bias[j];
        if (relu) x = fmaxf(x, 0.0f);
        if (add_aux_last) x += bias[j];
        op[(h + j) * so_n] = x;
      }
    }
  }
}

// Copies the (up to) 32 final output values of one row chunk, just stored at
// `op` = out + off by this thread, to every peer output at the same offset.
__device__ __forceinline__ void copy_to_peers(TcParams const &p, float const *op, int64_t off, int64_t nb,
                                              int64_t so_n) {
  const int64_t rem = p.n_size - nb;
  const int lim = rem < 32 ? (int)rem : 32;
  if (so_n == 1 && lim == 32 && ((reinterpret_cast<uintptr_t>(op) & 15) == 0)) {
    // the row's 32 values are contiguous: 16-byte vectors (a warp's lanes
    // hold different rows, so 4-byte stores would each be a separate write
    // over NVLink)
    float4 x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = reinterpret_cast<float4 const *>(op)[j];
    for (int i = 0; i < p.peers.n; ++i) {
      float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.peers.ptr[i]) + off);
      if (reinterpret_cast<uintptr_t>(dst) & 15) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float *d = reinterpret_cast<float *>(dst) + 4 * j;
          d[0] = x[j].x;
          d[1] = x[j].y;
          d[2] = x[j].z;
          d[3] = x[j].w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) dst[j] = x[j];
      }
    }
    return;
  }
  float x[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) x[j] = j < lim ? op[j * so_n] : 0.0f;
  for (int i = 0; i < p.peers.n; ++i) {
    float *dst = static_cast<float *>(p.peers.ptr[i]) + off;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < lim) dst[j * so_n] = x[j];
  }
}

// Writes 32 consecutive accumulator columns (output columns nb .. nb+31) of one
// output row with the fused first / last touch. `op` / `ap` point at column nb
// of the output / aux row; the full-chunk fast paths walk them by increments.
__device__ __forceinline__ void store_chunk(TcParams const &p, uint32_t const (&v)[32], float *op,
                                            const float *ap, int64_t nb, int64_t so_n, int64_t sa_n,
                                            int fast) {
  const bool relu = p.last_touch == 1;
  if (fast == 0 && nb + 32 <= p.n_size) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      *op = __uint_as_float(v[j]);
      op += so_n;
    }
  } else if (fast == 1 && nb + 32 <= p.n_size) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float x = __uint_as_float(v[j]) + __ldg(ap);
      *op = relu ? fmaxf(x, 0.0f) : x;
      op += so_n;
      ap += sa_n;
    }
  } else {
#pragma unroll 4
    for (int j = 0; j < 32; ++j) {
      if (nb + j < p.n_size) {
        float x = __uint_as_float(v[j]);
        if (p.first_touch == 3 /*COPY*/) x += *ap;
        else if (p.first_touch == 2 /*ADD*/) x += *op + *ap;
        else if (p.first_touch != 0 /*not ZERO*/) x += *op;
        if (p.last_touch == 1 /*RELU*/) x = fmaxf(x, 0.0f);
        else if (p.last_touch == 2 /*ADD*/) x += *ap;
        *op = x;
      }
      op += so_n;
      ap += sa_n;
    }
  }
}

}  // namespace eir
