// Internal plan objects behind the opaque `eir_plan` handle of the C-ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>
#include "eir_params.h"
#include "eir_cuda.h"

namespace eir {

// one loop dim after lowering (element strides)
struct LDim {
  int type = 0;
  int64_t size = 1;
  int64_t sl = 0, sr = 0, so = 0, sa = 0;
};

// a rank-5 TMA map with the data pointer bound at run time
struct MapSpec {
  int rank = 5;
  uint64_t dims[5] = {1, 1, 1, 1, 1};
  uint64_t strides_bytes[4] = {16, 16, 16, 16};  // strides of dims 1..4
  uint32_t box[5] = {1, 1, 1, 1, 1};
  CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B;
};

struct TensorMapCache {
  void const *ptr = nullptr;
  CUtensorMap map;
};

// helpers defined in eir_capi.cu
int api_set_error(int code, char const *msg);
int api_cuda_fail(cudaError_t e, char const *where);
int api_encode_map(MapSpec const &s, void const *ptr, CUtensorMap *m);
void api_count_launch();

}  // namespace eir

struct eir_plan;
namespace eir {
// launches the tensor-core kernel a plan chose (DMMA, CTA-pair tcgen05 or one-CTA tcgen05)
cudaError_t api_launch_tc(eir_plan const *p, CUtensorMap const &ma, CUtensorMap const &mb,
                          TcParams const &tp, void const *aux, void *out, int num_sms,
                          cudaStream_t st);
// One contraction on `stream` (eir_contract and its variants). ws: the plan's
// workspace of ws_bytes, or null for the plan's own (allocated on first use);
// err: the device error word for the bounded waits, or null for the
// device's own; peers / slab_ctr as for eir_contract_peers / _gather.
int api_contract(eir_plan *p, void const *l, void const *r, void const *aux, void *out,
                 PeerOutputs const *peers, void *stream, uint32_t *slab_ctr, void *ws, uint32_t *err,
                 int num_sms);
// the workspace bytes a call with these operands uses (0 when it takes the
// CUDA-core path, which reads the operands in place)
int64_t api_workspace_needed(eir_plan const *p, void const *l, void const *r);
// device address of the error word of eir_contract_no_alloc's static scratch
// on device `dev`, or null before that entry point's first call there
uint32_t *noalloc_error_word(int dev);
// a split-K plan (TcParams::split_k > 1): slices into the workspace `ws`,
// then the reduction into `out` with the plan's touches and peers
int api_launch_tc_split(eir_plan const *p, CUtensorMap const &ma, CUtensorMap const &mb,
                        TcParams const &tp, void const *aux, void *out, float *ws, int num_sms,
                        cudaStream_t st);
}  // namespace eir

struct eir_plan {
  int what = 0;  // 1 = contraction, 2 = permute
  int family = EIR_FAMILY_NONE;
  int64_t num_ops = 0;
  std::string text;

  // ---- contraction
  int dt_l = 0, dt_r = 0, dt_o = 0, comp = 0, first = 99, last = 99;
  int desc_flags = 0;
  bool empty = false;            // nothing to compute (a C/M/N dim of size 0)
  bool swapped = false;          // left and right change roles (dims and dt_l / dt_r are the swapped ones)
  std::vector<eir::LDim> dims;   // after size-1 removal and fusion
  eir::SimtParams simt;
  eir::DirectParams direct;      // the CUDA-core path of tiny problems (one output per thread)
  bool simt_direct = false;      // the CUDA-core path takes `direct`, not the tiled `simt`
  bool tc = false;
  // complex contraction: the right operand is expanded into real blocks
  // (cpx_expand, into the workspace) and `cpx_inner` contracts the real problem
  eir_plan *cpx_inner = nullptr;
  eir::PermuteParams cpx_expand;
  int64_t cpx_stride_right = 0;
  int tc_kind = 0, tc_bn = 128, tc_ksub = 1;
  bool tc_pair = false;  // CTA-pair (cta_group::2) kernel, 256-row tiles
  bool a_mn = false, b_mn = false;
  eir::TcParams tcp{};
  eir::MapSpec map_a, map_b;
  int tc_esize = 2;
  std::mutex mu;                 // guards the tensor-map caches
  eir::TensorMapCache cache_a, cache_b;

  // operand copies into the plan's workspace before the kernel: the operand
  // whose K walk disagrees is re-laid out (prepack: 0 = left, 1 = right,
  // -1 = none), and with TF32 compute both operands are rounded to TF32 on
  // the way; pre_l / pre_r are the copies' permute plans (null: read in place)
  int prepack = -1;
  eir_plan *pre_l = nullptr, *pre_r = nullptr;
  int64_t ws_off_l = 0, ws_off_r = 0;  // the copies' byte offsets in the workspace
  void *ws = nullptr;
  int64_t ws_bytes = 0;
  int64_t split_ws_offset = 0;  // split-K partial tiles: ws + this offset
  int ws_device = -1;

  // ---- output gather (eir_contract_gather)
  bool out_dense = false;         // the output is one contiguous block of out_elems
  int64_t out_elems = 0;
  // the output in slabs of its outermost dim when that dim is the kernel's
  // slowest tile loop (tiles then finish slab by slab), else one slab
  int64_t slab_count = 1;
  int64_t slab_elems = 0;
  int slab_loop = -1;             // tile loop of the slabs
  bool slab_counted = false;      // the kernel counts each slab's finished tiles
  uint32_t slab_target = 1;       // count of a finished slab
  // per-plan gather resources, created on first use on gather_device
  int gather_device = -1;
  uint32_t *slab_ctr = nullptr;
  cudaStream_t gather_streams[eir::kMaxPeers] = {};
  cudaEvent_t gather_start = nullptr;
  cudaEvent_t gather_done[eir::kMaxPeers] = {};

  // ---- permute (unary COPY) or unary ZERO
  eir::PermuteParams perm;
  bool unary_zero = false;
  int esize = 4;

  // ---- main-kernel timing (eir_plan_profile)
  bool profile = false;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> prof_events;
  size_t prof_used = 0;
};
