// Kernel parameter blocks shared by the planner (host) and the kernels.
// All strides are in elements.
#pragma once

#include <cstdint>

namespace eir {

constexpr int kMaxGroupDims = 6;   // dims per C/M/N/K group in the SIMT kernel
constexpr int kMaxPermDims = 8;    // dims of a permute after fusion

// A group of loop dimensions flattened into one index; dim 0 varies fastest.
struct GroupDims {
  int32_t n = 0;
  int32_t pad_ = 0;
  int64_t total = 1;
  int64_t size[kMaxGroupDims] = {};
  int64_t sl[kMaxGroupDims] = {};   // left strides
  int64_t sr[kMaxGroupDims] = {};   // right strides
  int64_t so[kMaxGroupDims] = {};   // out strides
  int64_t sa[kMaxGroupDims] = {};   // out_aux strides
};

constexpr int kMaxPeers = 7;

// Copies of the output on other GPUs (peer memory mapped into this process):
// the epilogue stores every final output element to `out` and, at the same
// element offset, to each peer output (an all-gather fused into the
// contraction; the stores cross NVLink while the next tiles compute).
struct PeerOutputs {
  int32_t n = 0;
  int32_t pad_ = 0;
  void *ptr[kMaxPeers] = {};
};

struct SimtParams {
  GroupDims c, m, n, k;
  int32_t first_touch;  // EIR_KTYPE_*
  int32_t last_touch;
  int32_t a_kfast;      // left: K is the fast (stride-1) direction -> load along K
  int32_t b_kfast;      // right: K is the fast direction
  int32_t round_tf32;   // TF32 compute: FP32 operands rounded to TF32 as they are loaded
  int32_t pad_;
  int64_t m_tiles, n_tiles;
  PeerOutputs peers;
};

// The direct CUDA-core contraction (one output element per thread) for tiny
// problems: the C, M and N dims form one output index (fastest output stride
// first), decomposed with 32-bit quotients q = mulhi64(x, magic), magic =
// ceil(2^64 / size), which is exact for x < 2^32 (Lemire, Kaser, Kurz,
// "Faster Remainder by Direct Computation", 2019); the planner only takes
// this kernel for fewer than 2^22 outputs. K runs as an inner loop over K
// dim 0 (fastest left stride) inside an outer loop over the other K dims.
constexpr int kMaxDirectDims = 3 * kMaxGroupDims;

struct DirectParams {
  int32_t nd = 0;            // output-index dims
  int32_t nk = 0;            // K dims
  int32_t first_touch = 0;   // EIR_KTYPE_*
  int32_t last_touch = 0;
  int32_t round_tf32 = 0;
  int32_t pad_ = 0;
  int64_t total = 0;         // output elements (< 2^22)
  int64_t k_inner = 1;       // size of K dim 0 (1 without K dims)
  int64_t k_outer = 1;       // product of the other K dims (0 when a K dim is empty)
  uint32_t size[kMaxDirectDims] = {};
  uint64_t magic[kMaxDirectDims] = {};   // ceil(2^64 / size); unused for size 1
  int64_t sl[kMaxDirectDims] = {};
  int64_t sr[kMaxDirectDims] = {};
  int64_t so[kMaxDirectDims] = {};
  int64_t sa[kMaxDirectDims] = {};
  uint32_t ksize[kMaxGroupDims] = {};
  uint64_t kmagic[kMaxGroupDims] = {};
  int64_t ksl[kMaxGroupDims] = {};
  int64_t ksr[kMaxGroupDims] = {};
  PeerOutputs peers;
};

// Permute: dims sorted so that dim 0 is the output's fastest dim.
struct PermuteParams {
  int32_t nd = 0;
  int32_t mode = 0;        // 0 = copy along the shared stride-1 dim, 1 = 2-D tile transpose
  int32_t vec = 1;         // elements per vector access (copy mode)
  int32_t tdim_in = 0;     // transpose: index of the input's fastest dim
  int32_t round_tf32 = 0;  // 32-bit elements rounded to the nearest TF32 value as they are copied
  int32_t pad_ = 0;
  int64_t size[kMaxPermDims] = {};
  int64_t sin[kMaxPermDims] = {};
  int64_t sout[kMaxPermDims] = {};
  int64_t total = 1;       // number of elements
  int64_t rows = 1;        // copy mode: number of rows (elements / size[0])
  int64_t batch = 1;       // transpose mode: number of (size[0] x size[tdim_in]) slices
};

// tcgen05 contraction. Operand tensor maps are 5-D; map dims 0/1 are the
// primitive (K / row) dims, dims 2..4 take their coordinate from `*_src`.
enum : int8_t {
  kSrcNone = 0,   // coordinate 0 (padding dim of size 1)
  kSrcKo0 = 1,
  kSrcKo1 = 2,
  kSrcLoop0 = 3,  // .. kSrcLoop0 + 3
};

constexpr int kMaxTileLoops = 4;

struct TcParams {
  int64_t m_size, n_size, kp_size;          // primitive M / N / K sizes
  int64_t so_m, so_n, sa_m, sa_n;           // out / aux strides of the primitive M and N dims
  int64_t loop_size[kMaxTileLoops];
  int64_t loop_so[kMaxTileLoops];
  int64_t loop_sa[kMaxTileLoops];
  int64_t ko_size[2];
  int64_t total_tiles;
  int32_t m_tiles, n_tiles, kp_blocks, k_steps;
  int32_t n_loops;
  int32_t group_m;                          // M tiles per raster group
  // ring stages per accumulation chunk (0 = the whole K walk in one chunk):
  // the tensor core's FP32 accumulation is biased over long K (about 2e-8
  // relative per accumulating MMA), so long K walks accumulate chunk by chunk
  // in TMEM and the epilogue adds the chunks in FP32 with rounding
  int32_t k_chunk;
  // split-K (one-CTA kernel): work item t is slice t / base_tiles of tile
  // t % base_tiles; slice s covers K stages [s n / split_k, (s+1) n / split_k)
  // and writes its partial tile into a dense FP32 workspace (out + s *
  // ws_slice), which a reduction kernel sums into the output
  int32_t split_k;
  int64_t base_tiles;
  int64_t ws_slice;
  int32_t first_touch, last_touch;
  int8_t a_src[5];
  int8_t b_src[5];
  int16_t pad_;
  uint32_t *err;                            // device error word
  PeerOutputs peers;
  // slab completion counters (eir_contract_gather; null otherwise): after
  // the final stores of a tile, every storing warp adds 1 to
  // slab_ctr[l[slab_loop]] (slab_ctr[0] when slab_loop < 0), so a copy
  // engine waiting for a slab's count can move that part of the output while
  // the kernel computes the next tiles
  uint32_t *slab_ctr;
  int32_t slab_loop;
  int32_t pad2_;
};

}  // namespace eir
