// CUDA-core kernels: the generic strided contraction (any layout, FP32/FP64
// accumulate, BF16/FP32/FP64 inputs) and the permute (Unary COPY) kernels.
//
// The generic contraction flattens each dim group (C, M, N, K) into one index
// and decomposes it with per-dim sizes/strides, so it reads every operand in
// place whatever its strides are; it is the path for contractions the tensor
// core lowering does not take (tiny trees, K = empty outer products, FP64
// until the DMMA kernel, unaligned strides). Semantics follow the reference's
// scalar loop engine: out = first_touch(out, aux); out += sum_K l*r;
// out = last_touch(out, aux) (ContractionBackendScalar.cpp:4-143,
// ContractionBackend.cpp:296-348,495-515, ContractionBackendTpp.cpp:130-163).
#include "eir_common.cuh"
#include "eir_params.h"
#include "eir_kernels.h"
#include "eir_launch.h"

namespace eir {

template <typename T>
__device__ __forceinline__ float to_f32(T x) {
  return static_cast<float>(x);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename TA, typename T>
__device__ __forceinline__ TA to_acc(T x) {
  return static_cast<TA>(to_f32(x));
}
template <>
__device__ __forceinline__ double to_acc<double, double>(double x) {
  return x;
}

// an operand value as the accumulation type, rounded to TF32 when the plan
// computes in TF32 (FP32 operands only)
template <typename TA, typename T>
__device__ __forceinline__ TA load_acc(T x, int32_t round_tf32) {
  return to_acc<TA>(x);
}
template <>
__device__ __forceinline__ float load_acc<float, float>(float x, int32_t round_tf32) {
  return round_tf32 ? __uint_as_float(round_tf32_bits(__float_as_uint(x))) : x;
}

__device__ __forceinline__ void decompose(GroupDims const &g, int64_t x, int64_t &ol, int64_t &orr,
                                          int64_t &oo, int64_t &oa) {
  ol = orr = oo = oa = 0;
#pragma unroll
  for (int d = 0; d < kMaxGroupDims; ++d) {
    if (d < g.n) {
      int64_t i = x % g.size[d];
      x /= g.size[d];
      ol += i * g.sl[d];
      orr += i * g.sr[d];
      oo += i * g.so[d];
      oa += i * g.sa[d];
    }
  }
}

constexpr int kSimtBM = 64, kSimtBN = 64, kSimtBK = 16;
constexpr int kSimtChunkK = 256;  // K per accumulation chunk (a multiple of kSimtBK)

template <typename TL, typename TR, typename TO, typename TA>
__global__ void __launch_bounds__(256)
    simt_contract_kernel(const SimtParams p, const TL *__restrict__ L, const TR *__restrict__ R,
                         const TO *__restrict__ AUX, TO *__restrict__ OUT) {
  constexpr int BM = kSimtBM, BN = kSimtBN, BK = kSimtBK;
  __shared__ TA As[BK][BM + 1];
  __shared__ TA Bs[BK][BN + 1];
  __shared__ int64_t row_l[BM], row_o[BM], row_a[BM];
  __shared__ int64_t col_r[BN], col_o[BN], col_a[BN];
  __shared__ int64_t k_l[BK], k_r[BK];

  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  int64_t bid = blockIdx.x;
  const int64_t mt = bid % p.m_tiles;
  bid /= p.m_tiles;
  const int64_t nt = bid % p.n_tiles;
  const int64_t ct = bid / p.n_tiles;

  const int64_t M = p.m.total, N = p.n.total, K = p.k.total;
  int64_t c_l, c_r, c_o, c_a;
  decompose(p.c, ct, c_l, c_r, c_o, c_a);

  if (tid < BM) {
    int64_t m = mt * BM + tid;
    int64_t ol = 0, orr, oo = 0, oa = 0;
    if (m < M) decompose(p.m, m, ol, orr, oo, oa);
    row_l[tid] = ol + c_l;
    row_o[tid] = oo + c_o;
    row_a[tid] = oa + c_a;
  } else if (tid < BM + BN) {
    int t = tid - BM;
    int64_t n = nt * BN + t;
    int64_t ol, orr = 0, oo = 0, oa = 0;
    if (n < N) decompose(p.n, n, ol, orr, oo, oa);
    col_r[t] = orr + c_r;
    col_o[t] = oo;
    col_a[t] = oa;
  }

  // acc: the current chunk of kSimtChunkK products; tot: the sum of the
  // chunks. Chunked accumulation keeps the rounding error of long K near
  // (sqrt(chunk) + sqrt(K / chunk)) ulp instead of sqrt(K) ulp.
  TA acc[4][4], tot[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = tot[i][j] = TA(0);

  for (int64_t k0 = 0; k0 < K; k0 += BK) {
    if (tid < BK) {
      int64_t k = k0 + tid;
      int64_t ol = 0, orr = 0, oo, oa;
      if (k < K) decompose(p.k, k, ol, orr, oo, oa);
      k_l[tid] = ol;
      k_r[tid] = orr;
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < (BM * BK) / 256; ++q) {
      int e = tid + 256 * q;
      int kk, mm;
      if (p.a_kfast) {
        kk = e % BK;
        mm = e / BK;
      } else {
        mm = e % BM;
        kk = e / BM;
      }
      int64_t m = mt * BM + mm, k = k0 + kk;
      As[kk][mm] = (m < M && k < K) ? load_acc<TA>(L[row_l[mm] + k_l[kk]], p.round_tf32) : TA(0);
    }
#pragma unroll
    for (int q = 0; q < (BN * BK) / 256; ++q) {
      int e = tid + 256 * q;
      int kk, nn;
      if (p.b_kfast) {
        kk = e % BK;
        nn = e / BK;
      } else {
        nn = e % BN;
        kk = e / BN;
      }
      int64_t n = nt * BN + nn, k = k0 + kk;
      Bs[kk][nn] = (n < N && k < K) ? load_acc<TA>(R[col_r[nn] + k_r[kk]], p.round_tf32) : TA(0);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      TA a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][tx + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][ty + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * b[j];
    }
    __syncthreads();
    if (((k0 + BK) % kSimtChunkK) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          tot[i][j] += acc[i][j];
          acc[i][j] = TA(0);
        }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) tot[i][j] += acc[i][j];

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int mm = tx + 16 * i;
    const int64_t m = mt * BM + mm;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int nn = ty + 16 * j;
      const int64_t n = nt * BN + nn;
      if (n >= N) continue;
      const int64_t o = row_o[mm] + col_o[nn];
      const int64_t a = row_a[mm] + col_a[nn];
      TA x = tot[i][j];
      if (p.first_touch == 3 /*COPY*/) x += static_cast<TA>(AUX[a]);
      else if (p.first_touch == 2 /*ADD*/) x += static_cast<TA>(OUT[o]) + static_cast<TA>(AUX[a]);
      else if (p.first_touch != 0 /*ZERO*/) x += static_cast<TA>(OUT[o]);
      if (p.last_touch == 1 /*RELU*/) x = x > TA(0) ? x : TA(0);
      else if (p.last_touch == 2 /*ADD*/) x += static_cast<TA>(AUX[a]);
      OUT[o] = static_cast<TO>(x);
      for (int q = 0; q < p.peers.n; ++q) static_cast<TO *>(p.peers.ptr[q])[o] = static_cast<TO>(x);
    }
  }
}

template <typename TL, typename TR, typename TO, typename TA>
static cudaError_t launch_simt_t(SimtParams const &p, void const *l, void const *r,
                                 void const *aux, void *out, cudaStream_t st) {
  int64_t blocks = p.m_tiles * p.n_tiles * p.c.total;
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  return launch_kernel(simt_contract_kernel<TL, TR, TO, TA>, dim3((unsigned)blocks), dim3(256), 0, st,
                       p, static_cast<TL const *>(l), static_cast<TR const *>(r),
                       static_cast<TO const *>(aux), static_cast<TO *>(out));
}

// dtypes: 0 = FP32, 1 = FP64, 2 = BF16 (values of the C-ABI enum)
cudaError_t launch_simt_contract(int dt_l, int dt_r, int dt_o, SimtParams const &p, void const *l,
                                 void const *r, void const *aux, void *out, cudaStream_t st) {
  if (dt_o == 1) {
    if (dt_l == 1 && dt_r == 1) return launch_simt_t<double, double, double, double>(p, l, r, aux, out, st);
    return cudaErrorInvalidValue;
  }
  if (dt_o != 0) return cudaErrorInvalidValue;
  if (dt_l == 0 && dt_r == 0) return launch_simt_t<float, float, float, float>(p, l, r, aux, out, st);
  if (dt_l == 2 && dt_r == 2)
    return launch_simt_t<__nv_bfloat16, __nv_bfloat16, float, float>(p, l, r, aux, out, st);
  if (dt_l == 2 && dt_r == 0)
    return launch_simt_t<__nv_bfloat16, float, float, float>(p, l, r, aux, out, st);
  if (dt_l == 0 && dt_r == 2)
    return launch_simt_t<float, __nv_bfloat16, float, float>(p, l, r, aux, out, st);
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------ direct kernel
// One output element per thread, for contractions too small to fill the 64 x
// 64 tiles above (trees of small tensors): the tiled kernel's fixed cost (a
// long, cold instruction stream per CTA) then dominates. Same semantics and
// chunked accumulation as the tiled kernel.
__device__ __forceinline__ uint32_t div_magic(uint32_t x, uint32_t size, uint64_t magic) {
  return size == 1u ? x : (uint32_t)__umul64hi((uint64_t)x, magic);
}

template <typename TL, typename TR, typename TO, typename TA>
__global__ void __launch_bounds__(256)
    simt_direct_kernel(const DirectParams p, const TL *__restrict__ L, const TR *__restrict__ R,
                       const TO *__restrict__ AUX, TO *__restrict__ OUT) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= p.total) return;
  uint32_t x = (uint32_t)gid;
  int64_t ol = 0, orr = 0, oo = 0, oa = 0;
#pragma unroll 1
  for (int d = 0; d < p.nd; ++d) {
    const uint32_t q = div_magic(x, p.size[d], p.magic[d]);
    const int64_t i = (int64_t)(x - q * p.size[d]);
    x = q;
    ol += i * p.sl[d];
    orr += i * p.sr[d];
    oo += i * p.so[d];
    oa += i * p.sa[d];
  }
  TA acc = TA(0), tot = TA(0);
  int chunk = 0;
  const int64_t s_l = p.ksl[0], s_r = p.ksr[0];
#pragma unroll 1
  for (int64_t j = 0; j < p.k_outer; ++j) {
    int64_t bl = ol, br = orr;
    uint32_t y = (uint32_t)j;
#pragma unroll 1
    for (int d = 1; d < p.nk; ++d) {
      const uint32_t q = div_magic(y, p.ksize[d], p.kmagic[d]);
      const int64_t i = (int64_t)(y - q * p.ksize[d]);
      y = q;
      bl += i * p.ksl[d];
      br += i * p.ksr[d];
    }
#pragma unroll 4
    for (int64_t i = 0; i < p.k_inner; ++i) {
      acc += load_acc<TA>(L[bl + i * s_l], p.round_tf32) * load_acc<TA>(R[br + i * s_r], p.round_tf32);
      if (++chunk == kSimtChunkK) {
        tot += acc;
        acc = TA(0);
        chunk = 0;
      }
    }
  }
  TA v = tot + acc;
  if (p.first_touch == 3 /*COPY*/) v += static_cast<TA>(AUX[oa]);
  else if (p.first_touch == 2 /*ADD*/) v += static_cast<TA>(OUT[oo]) + static_cast<TA>(AUX[oa]);
  else if (p.first_touch != 0 /*ZERO*/) v += static_cast<TA>(OUT[oo]);
  if (p.last_touch == 1 /*RELU*/) v = v > TA(0) ? v : TA(0);
  else if (p.last_touch == 2 /*ADD*/) v += static_cast<TA>(AUX[oa]);
  OUT[oo] = static_cast<TO>(v);
  for (int q = 0; q < p.peers.n; ++q) static_cast<TO *>(p.peers.ptr[q])[oo] = static_cast<TO>(v);
}

template <typename TL, typename TR, typename TO, typename TA>
static cudaError_t launch_direct_t(DirectParams const &p, void const *l, void const *r, void const *aux,
                                   void *out, cudaStream_t st) {
  if (p.total <= 0) return cudaSuccess;
  if (p.total >= (int64_t(1) << 32)) return cudaErrorInvalidConfiguration;
  const int64_t blocks = (p.total + 255) / 256;
  return launch_kernel(simt_direct_kernel<TL, TR, TO, TA>, dim3((unsigned)blocks), dim3(256), 0, st, p,
                       static_cast<TL const *>(l), static_cast<TR const *>(r), static_cast<TO const *>(aux),
                       static_cast<TO *>(out));
}

cudaError_t launch_simt_direct(int dt_l, int dt_r, int dt_o, DirectParams const &p, void const *l,
                               void const *r, void const *aux, void *out, cudaStream_t st) {
  if (dt_o == 1) {
    if (dt_l == 1 && dt_r == 1) return launch_direct_t<double, double, double, double>(p, l, r, aux, out, st);
    return cudaErrorInvalidValue;
  }
  if (dt_o != 0) return cudaErrorInvalidValue;
  if (dt_l == 0 && dt_r == 0) return launch_direct_t<float, float, float, float>(p, l, r, aux, out, st);
  if (dt_l == 2 && dt_r == 2)
    return launch_direct_t<__nv_bfloat16, __nv_bfloat16, float, float>(p, l, r, aux, out, st);
  if (dt_l == 2 && dt_r == 0)
    return launch_direct_t<__nv_bfloat16, float, float, float>(p, l, r, aux, out, st);
  if (dt_l == 0 && dt_r == 2)
    return launch_direct_t<float, __nv_bfloat16, float, float>(p, l, r, aux, out, st);
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------ permute
// an element as copied by a permute: FP32 words rounded to the nearest TF32
// value when the permute feeds a TF32 contraction (PermuteParams::round_tf32)
template <typename T>
__device__ __forceinline__ T copy_elem(T x, int32_t round_tf32) {
  return x;
}
template <>
__device__ __forceinline__ uint32_t copy_elem<uint32_t>(uint32_t x, int32_t round_tf32) {
  return round_tf32 ? round_tf32_bits(x) : x;
}

// copy mode: dim 0 is stride-1 in input and output; V elements per access.
// ZERO: the unary ZERO primitive (out = 0 over the output's strides; `in` unused).
// I: index type, int32_t whenever every element offset of both tensors fits.
// A copy whose dims all fused into one (nd == 1: a contiguous or uniformly
// strided run, e.g. the TF32-rounding copy of an operand) skips the index
// decomposition and keeps 4 independent vectors in flight per thread.
template <typename T, int V, bool ZERO, typename I>
__global__ void __launch_bounds__(256)
    permute_copy_kernel(const PermuteParams p, const T *__restrict__ in, T *__restrict__ out) {
  struct alignas(sizeof(T) * V) Vec {
    T v[V];
  };
  pdl_launch_dependents();
  pdl_wait();
  const I n0v = (I)(p.size[0] / V);
  const I total = (I)p.rows * n0v;
  const I nthr = (I)gridDim.x * (I)blockDim.x;
  const I tid = (I)blockIdx.x * (I)blockDim.x + (I)threadIdx.x;
  if (p.nd == 1) {
    const I sin0 = (I)p.sin[0], sout0 = (I)p.sout[0];
    for (I g = tid; g < total; g += 4 * nthr) {
      Vec v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const I e = g + (I)j * nthr;
        if (!ZERO && e < total) v[j] = *reinterpret_cast<Vec const *>(in + e * V * sin0);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const I e = g + (I)j * nthr;
        if (e >= total) continue;
        if (ZERO) {
          *reinterpret_cast<Vec *>(out + e * V * sout0) = Vec{};
        } else {
#pragma unroll
          for (int k = 0; k < V; ++k) v[j].v[k] = copy_elem(v[j].v[k], p.round_tf32);
          *reinterpret_cast<Vec *>(out + e * V * sout0) = v[j];
        }
      }
    }
    return;
  }
  // general: 4 vectors per thread and iteration, each decomposed into its row
  // offsets (V > 1 only when dim 0 has unit stride on both sides, checked by
  // the planner)
  for (I g = tid; g < total; g += 4 * nthr) {
    I src[4], dst[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const I e = g + (I)j * nthr;
      I i0 = e % n0v, row = e / n0v;
      I oi = i0 * V * (I)p.sin[0], oo = i0 * V * (I)p.sout[0];
#pragma unroll
      for (int d = 1; d < kMaxPermDims; ++d) {
        if (d < p.nd) {
          I i = row % (I)p.size[d];
          row /= (I)p.size[d];
          oi += i * (I)p.sin[d];
          oo += i * (I)p.sout[d];
        }
      }
      src[j] = oi;
      dst[j] = oo;
    }
    Vec v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (!ZERO && g + (I)j * nthr < total) v[j] = *reinterpret_cast<Vec const *>(in + src[j]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (g + (I)j * nthr >= total) continue;
      if (ZERO) {
        *reinterpret_cast<Vec *>(out + dst[j]) = Vec{};
      } else {
#pragma unroll
        for (int k = 0; k < V; ++k) v[j].v[k] = copy_elem(v[j].v[k], p.round_tf32);
        *reinterpret_cast<Vec *>(out + dst[j]) = v[j];
      }
    }
  }
}

// transpose mode: dim 0 is the output's stride-1 dim, dim tdim_in the input's.
// 64 x 64 tiles through shared memory (padded rows: conflict-free both ways),
// 16 elements per thread in flight on each side, so the copy is not latency
// bound. I: index type, int32_t whenever every element offset of both tensors
// fits (the common case; 64-bit divisions in the tile decode are slow).
constexpr int kTransposeTile = 64;
template <typename T, typename I>
__global__ void __launch_bounds__(256)
    permute_transpose_kernel(const PermuteParams p, const T *__restrict__ in, T *__restrict__ out) {
  constexpr int TS = kTransposeTile;
  __shared__ T tile[TS][TS + 1];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  const int td = p.tdim_in;
  pdl_launch_dependents();
  pdl_wait();
  const I s0 = (I)p.size[0], st = (I)p.size[td];
  const I t0 = (s0 + TS - 1) / TS, tt = (st + TS - 1) / TS;
  const I nblk = t0 * tt * (I)p.batch;
  const I sin0 = (I)p.sin[0], sint = (I)p.sin[td], sout0 = (I)p.sout[0], soutt = (I)p.sout[td];
  for (I blk = (I)blockIdx.x; blk < nblk; blk += (I)gridDim.x) {
    // diagonal order: blocks running at the same time cover different tiles
    // along both dims, not one band of columns of the input (which maps to few
    // DRAM channels); b0 -> bt is a rotation, so every tile is visited once
    const I b0 = blk % t0;
    const I r = blk / t0;
    const I bt = (r % tt + b0) % tt;
    I bat = r / tt;
    I oi = 0, oo = 0;
#pragma unroll
    for (int d = 1; d < kMaxPermDims; ++d) {
      if (d < p.nd && d != td) {
        const I i = bat % (I)p.size[d];
        bat /= (I)p.size[d];
        oi += i * (I)p.sin[d];
        oo += i * (I)p.sout[d];
      }
    }
    // load: consecutive threads walk the input's stride-1 dim (2 x 32 columns)
#pragma unroll
    for (int i = 0; i < TS / 8; ++i)
#pragma unroll
      for (int c = 0; c < TS / 32; ++c) {
        const I it = bt * TS + tx + 32 * c, i0 = b0 * TS + ty + 8 * i;
        if (it < st && i0 < s0)
          tile[ty + 8 * i][tx + 32 * c] = copy_elem(in[oi + it * sint + i0 * sin0], p.round_tf32);
      }
    __syncthreads();
    // store: consecutive threads walk the output's stride-1 dim
#pragma unroll
    for (int i = 0; i < TS / 8; ++i)
#pragma unroll
      for (int c = 0; c < TS / 32; ++c) {
        const I i0 = b0 * TS + tx + 32 * c, it = bt * TS + ty + 8 * i;
        if (it < st && i0 < s0) out[oo + i0 * sout0 + it * soutt] = tile[tx + 32 * c][ty + 8 * i];
      }
    __syncthreads();
  }
}

// largest element offset of a permute's input or output (non-negative strides)
static bool offsets_fit_int32(PermuteParams const &p) {
  int64_t span_in = 0, span_out = 0;
  for (int d = 0; d < p.nd; ++d) {
    if (p.sin[d] < 0 || p.sout[d] < 0) return false;
    span_in += (p.size[d] - 1) * p.sin[d];
    span_out += (p.size[d] - 1) * p.sout[d];
  }
  return span_in < (int64_t(1) << 31) - 1 && span_out < (int64_t(1) << 31) - 1 &&
         p.total < (int64_t(1) << 31);
}

// complex contraction operand: B' = [[Br, Bi], [-Bi, Br]] as four packed real
// blocks (block ci * 2 + co at offset (ci * 2 + co) * nb); p describes B's
// non-complex dims (sizes, source strides, packed destination strides)
template <typename T>
__global__ void __launch_bounds__(256)
    cpx_expand_kernel(const PermuteParams p, int64_t cpx_stride, const T *__restrict__ in,
                      T *__restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t nb = p.total;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nb;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = e, oi = 0, oo = 0;
#pragma unroll
    for (int d = 0; d < kMaxPermDims; ++d) {
      if (d < p.nd) {
        const int64_t i = r % p.size[d];
        r /= p.size[d];
        oi += i * p.sin[d];
        oo += i * p.sout[d];
      }
    }
    const T re = in[oi], im = in[oi + cpx_stride];
    out[oo] = re;
    out[nb + oo] = im;
    out[2 * nb + oo] = -im;
    out[3 * nb + oo] = re;
  }
}

cudaError_t launch_cpx_expand(int esize, PermuteParams const &p, int64_t cpx_stride, void const *in,
                              void *out, int num_sms, cudaStream_t st) {
  if (p.total == 0) return cudaSuccess;
  int64_t blocks = (p.total + 255) / 256;
  if (blocks > (int64_t)num_sms * 16) blocks = (int64_t)num_sms * 16;
  if (esize == 4)
    return launch_kernel(cpx_expand_kernel<float>, dim3((unsigned)blocks), dim3(256), 0, st, p,
                         cpx_stride, static_cast<float const *>(in), static_cast<float *>(out));
  if (esize == 8)
    return launch_kernel(cpx_expand_kernel<double>, dim3((unsigned)blocks), dim3(256), 0, st, p,
                         cpx_stride, static_cast<double const *>(in), static_cast<double *>(out));
  return cudaErrorInvalidValue;
}

template <typename T, bool ZERO, typename I>
static cudaError_t launch_copy_t(PermuteParams const &p, T const *i, T *o, int64_t blocks, cudaStream_t st) {
  const dim3 g((unsigned)blocks), b(256);
  switch (p.vec) {
    case 1: return launch_kernel(permute_copy_kernel<T, 1, ZERO, I>, g, b, 0, st, p, i, o);
    case 2: return launch_kernel(permute_copy_kernel<T, 2, ZERO, I>, g, b, 0, st, p, i, o);
    case 4: return launch_kernel(permute_copy_kernel<T, 4, ZERO, I>, g, b, 0, st, p, i, o);
    case 8: return launch_kernel(permute_copy_kernel<T, 8, ZERO, I>, g, b, 0, st, p, i, o);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static cudaError_t launch_permute_t(PermuteParams const &p, void const *in, void *out, int num_sms,
                                    bool zero, cudaStream_t st) {
  if (p.total == 0) return cudaSuccess;
  const T *i = static_cast<T const *>(in);
  T *o = static_cast<T *>(out);
  cudaError_t e = cudaSuccess;
  if (zero && p.mode != 0) return cudaErrorInvalidValue;  // ZERO plans are row plans
  if (p.mode == 0) {
    int64_t work = p.total / p.vec;
    int64_t blocks = (work + 255) / 256;
    int64_t cap = (int64_t)num_sms * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    if (offsets_fit_int32(p))
      e = zero ? launch_copy_t<T, true, int32_t>(p, i, o, blocks, st)
               : launch_copy_t<T, false, int32_t>(p, i, o, blocks, st);
    else
      e = zero ? launch_copy_t<T, true, int64_t>(p, i, o, blocks, st)
               : launch_copy_t<T, false, int64_t>(p, i, o, blocks, st);
  } else {
    const int64_t ts = kTransposeTile;
    int64_t nblk = ((p.size[0] + ts - 1) / ts) * ((p.size[p.tdim_in] + ts - 1) / ts) * p.batch;
    int64_t cap = (int64_t)num_sms * 8;  // 8 x 256 threads per SM
    int64_t blocks = nblk < cap ? nblk : cap;
    if (blocks < 1) blocks = 1;
    if (offsets_fit_int32(p))
      e = launch_kernel(permute_transpose_kernel<T, int32_t>, dim3((unsigned)blocks), dim3(256), 0, st,
                        p, i, o);
    else
      e = launch_kernel(permute_transpose_kernel<T, int64_t>, dim3((unsigned)blocks), dim3(256), 0, st,
                        p, i, o);
  }
  return e;
}

cudaError_t launch_permute(int esize, PermuteParams const &p, void const *in, void *out,
                           int num_sms, cudaStream_t st, bool zero) {
  switch (esize) {
    case 2: return launch_permute_t<uint16_t>(p, in, out, num_sms, zero, st);
    case 4: return launch_permute_t<uint32_t>(p, in, out, num_sms, zero, st);
    case 8: return launch_permute_t<uint64_t>(p, in, out, num_sms, zero, st);
    default: return cudaErrorInvalidValue;
  }
}

// Sets every slab counter of a gathered contraction to its final value once
// the contraction kernel before it in the stream has completed (launched
// without programmatic serialisation, so it starts only after that kernel and
// its memory writes are complete): every copy that waits for a slab's count
// is then released, even if the kernel counted fewer tiles (a kernel family
// that does not count, or one that stopped after a bounded wait gave up).
__global__ void slab_release_kernel(uint32_t *ctr, int32_t n, uint32_t value) {
  for (int32_t i = threadIdx.x; i < n; i += blockDim.x) atomicMax(ctr + i, value);
}

cudaError_t launch_slab_release(uint32_t *ctr, int32_t n, uint32_t value, cudaStream_t st) {
  slab_release_kernel<<<1, 128, 0, st>>>(ctr, n, value);
  return cudaGetLastError();
}

}  // namespace eir
