// C-ABI of the einsum_ir B200 backend: planning (lowering of a strided binary
// contraction or permute to one of the kernel families) and launches.
//
// Lowering, in the spirit of the reference's ContractionOptimizer
// (ContractionOptimizer.cpp:47-111: drop size-1 loops, fuse contiguous loops)
// but with B200 targets instead of CPU GEMM leaves:
//   1. size-1 dims are dropped; dims of one type whose strides are contiguous
//      in every tensor are fused;
//   2. tensor-core path (BF16, TF32, 3xTF32): choose a primitive K dim that is
//      stride-1 in a K-major operand (or any K dim if both operands are
//      MN-major), the primitive M / N dims (the output's fastest M dim), map
//      the other K dims to up to two outer K loops and the other C / M / N dims
//      to up to four tile loops, and describe each operand as a 5-D TMA map
//      over its native strides. If both operands are K-major with different
//      stride-1 K dims the smaller operand is pre-permuted into a workspace
//      (the reference packs with a transpose for the same reason,
//      ContractionOptimizer.cpp:337-447);
//   3. otherwise the generic SIMT kernel reads the operands in place.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>
#include "eir_kernels.h"
#include "eir_plan.h"

using eir::LDim;

namespace {

thread_local std::string g_last_error;
std::atomic<int64_t> g_launches{0};

int set_error(int code, std::string const &msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, char const *where) {
  return set_error(EIR_CUDA_ERROR, std::string(where) + ": " + cudaGetErrorString(e));
}

// ---- per-device state: SM count, device error word
struct DeviceState {
  int num_sms = 0;
  uint32_t *err = nullptr;
};
std::mutex g_dev_mu;
DeviceState g_dev[64];

int device_state(DeviceState **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return set_error(EIR_CUDA_ERROR, "device index out of range");
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceState &d = g_dev[dev];
  if (d.num_sms == 0) {
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    e = cudaMalloc(&d.err, sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(error word)");
    e = cudaMemset(d.err, 0, sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(error word)");
    d.num_sms = n;
  }
  *out = &d;
  return EIR_SUCCESS;
}

// ---- driver entry point for tensor-map encoding (no link against libcuda)
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encoder() {
  std::call_once(g_encode_once, []() {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr) return set_error(EIR_CUDA_ERROR, "cuTensorMapEncodeTiled unavailable");
  return EIR_SUCCESS;
}

int encode_map(eir::MapSpec const &s, void const *ptr, CUtensorMap *m) {
  int rc = get_encoder();
  if (rc != EIR_SUCCESS) return rc;
  uint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(m, s.dtype, s.rank, const_cast<void *>(ptr), s.dims, s.strides_bytes, s.box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, s.swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(EIR_CUDA_ERROR, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return EIR_SUCCESS;
}

int64_t dtype_bytes(int dt) {
  switch (dt) {
    case EIR_FP32: return 4;
    case EIR_FP64: return 8;
    case EIR_BF16: return 2;
    default: return -1;
  }
}

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

char const *type_name(int t) {
  switch (t) {
    case EIR_DIM_C: return "C";
    case EIR_DIM_M: return "M";
    case EIR_DIM_N: return "N";
    case EIR_DIM_K: return "K";
    default: return "?";
  }
}

// drop size-1 dims and fuse dims of one type that are contiguous in every tensor
std::vector<LDim> simplify_dims(std::vector<LDim> d) {
  d.erase(std::remove_if(d.begin(), d.end(), [](LDim const &x) { return x.size == 1; }), d.end());
  bool changed = true;
  while (changed) {
    changed = false;
    for (size_t i = 0; i < d.size() && !changed; ++i) {
      for (size_t o = 0; o < d.size() && !changed; ++o) {
        if (i == o || d[i].type != d[o].type) continue;
        LDim const &in = d[i];
        LDim const &ou = d[o];
        if (ou.sl == in.sl * in.size && ou.sr == in.sr * in.size && ou.so == in.so * in.size &&
            ou.sa == in.sa * in.size) {
          LDim f = in;
          f.size = in.size * ou.size;
          d[i] = f;
          d.erase(d.begin() + o);
          changed = true;
        }
      }
    }
  }
  return d;
}

int build_group(std::vector<LDim> const &dims, int type, eir::GroupDims *g) {
  std::vector<LDim> sel;
  for (auto const &x : dims)
    if (x.type == type) sel.push_back(x);
  if ((int)sel.size() > eir::kMaxGroupDims) return -1;
  // fastest index first: order by the stride that matters for coalescing
  std::stable_sort(sel.begin(), sel.end(), [type](LDim const &a, LDim const &b) {
    int64_t ka = (type == EIR_DIM_K) ? std::llabs(a.sl) : std::llabs(a.so);
    int64_t kb = (type == EIR_DIM_K) ? std::llabs(b.sl) : std::llabs(b.so);
    return ka < kb;
  });
  g->n = (int)sel.size();
  g->total = 1;
  for (int i = 0; i < g->n; ++i) {
    g->size[i] = sel[i].size;
    g->sl[i] = sel[i].sl;
    g->sr[i] = sel[i].sr;
    g->so[i] = sel[i].so;
    g->sa[i] = sel[i].sa;
    g->total *= sel[i].size;
  }
  return 0;
}

int64_t min_abs_stride(std::vector<LDim> const &dims, int type, bool left) {
  int64_t m = INT64_MAX;
  for (auto const &x : dims)
    if (x.type == type) m = std::min<int64_t>(m, std::llabs(left ? x.sl : x.sr));
  return m;
}

int64_t env_int(char const *name, int64_t dflt) {
  char const *v = std::getenv(name);
  if (v == nullptr || *v == 0) return dflt;
  return std::atoll(v);
}

// ceil(2^64 / d) for 2 <= d < 2^32: the multiplier of div_magic (kernels_simt.cu)
uint64_t magic_of(int64_t d) { return d >= 2 ? UINT64_MAX / (uint64_t)d + 1 : 0; }

// The direct CUDA-core kernel's parameters (eir::DirectParams) from the
// plan's dims and SIMT groups. The CUDA-core path takes it for tiny problems:
// fewer than 2^22 outputs (the 32-bit index decomposition) and a short K
// walk per output (K <= 64, or outputs x K <= 2^16). EIR_SIMT_DIRECT=0 keeps
// the tiled kernel.
void build_direct(eir_plan *p) {
  eir::DirectParams &d = p->direct;
  d = eir::DirectParams{};
  std::vector<LDim> od;
  for (auto const &x : p->dims)
    if (x.type != EIR_DIM_K) od.push_back(x);
  if ((int)od.size() > eir::kMaxDirectDims) return;
  std::stable_sort(od.begin(), od.end(),
                   [](LDim const &a, LDim const &b) { return std::llabs(a.so) < std::llabs(b.so); });
  int64_t total = 1;
  for (auto const &x : od) total *= x.size;
  const eir::GroupDims &k = p->simt.k;
  const int64_t k_total = k.total;
  const bool small = total < (int64_t(1) << 22) &&
                     (k_total <= 64 || (double)total * (double)k_total <= (double)(1 << 16));
  if (!small || env_int("EIR_SIMT_DIRECT", 1) == 0) return;
  d.nd = (int32_t)od.size();
  for (int i = 0; i < d.nd; ++i) {
    d.size[i] = (uint32_t)od[i].size;
    d.magic[i] = magic_of(od[i].size);
    d.sl[i] = od[i].sl;
    d.sr[i] = od[i].sr;
    d.so[i] = od[i].so;
    d.sa[i] = od[i].sa;
  }
  d.nk = k.n;
  for (int i = 0; i < k.n; ++i) {
    d.ksize[i] = (uint32_t)k.size[i];
    d.kmagic[i] = magic_of(k.size[i]);
    d.ksl[i] = k.sl[i];
    d.ksr[i] = k.sr[i];
  }
  d.total = total;
  if (k_total == 0) {
    d.k_inner = 0;
    d.k_outer = 0;
  } else {
    d.k_inner = k.n > 0 ? k.size[0] : 1;
    d.k_outer = k_total / d.k_inner;
  }
  d.first_touch = p->simt.first_touch;
  d.last_touch = p->simt.last_touch;
  d.round_tf32 = p->simt.round_tf32;
  p->simt_direct = true;
}

// Permute planning shared by eir_permute_plan_create and operand pre-packing.
int plan_permute(int nd, int64_t const *sizes, int64_t const *sin, int64_t const *sout, int esize,
                 eir::PermuteParams *pp, std::string *text) {
  std::vector<LDim> d;
  for (int i = 0; i < nd; ++i) {
    if (sizes[i] < 0) return set_error(EIR_INVALID_ARGUMENT, "negative permute size");
    LDim x;
    x.type = 0;
    x.size = sizes[i];
    x.sl = sin[i];
    x.so = sout[i];
    d.push_back(x);
  }
  int64_t total = 1;
  for (auto const &x : d) total *= x.size;
  d = simplify_dims(d);
  *pp = eir::PermuteParams();
  pp->total = total;
  if (total == 0 || d.empty()) {
    // scalar (all dims size 1) or empty tensor
    pp->nd = 1;
    pp->size[0] = total == 0 ? 0 : 1;
    pp->sin[0] = 1;
    pp->sout[0] = 1;
    pp->rows = 1;
    pp->mode = 0;
    pp->vec = 1;
    if (text) *text = "permute: scalar/empty";
    return EIR_SUCCESS;
  }
  if ((int)d.size() > eir::kMaxPermDims)
    return set_error(EIR_COMPILATION_FAILED, "permute has too many non-fusable dims");
  // dim 0 = the output's fastest dim
  std::stable_sort(d.begin(), d.end(),
                   [](LDim const &a, LDim const &b) { return std::llabs(a.so) < std::llabs(b.so); });
  int tin = 0;
  for (int i = 1; i < (int)d.size(); ++i)
    if (std::llabs(d[i].sl) < std::llabs(d[tin].sl)) tin = i;
  pp->nd = (int)d.size();
  for (int i = 0; i < pp->nd; ++i) {
    pp->size[i] = d[i].size;
    pp->sin[i] = d[i].sl;
    pp->sout[i] = d[i].so;
  }
  if (tin == 0 || d[0].so != 1 || d[tin].sl != 1) {
    // shared fastest dim (or no unit strides at all): row copy
    pp->mode = 0;
    int vec = 1;
    if (d[0].so == 1 && d[0].sl == 1) {
      vec = (int)(16 / esize);
      while (vec > 1) {
        bool ok = d[0].size % vec == 0;
        for (int i = 1; i < pp->nd; ++i) ok = ok && (d[i].sl % vec == 0) && (d[i].so % vec == 0);
        if (ok) break;
        vec /= 2;
      }
    } else if (tin != 0) {
      // no unit stride on one side: still correct with the generic row copy;
      // put the dims in the row decomposition by treating dim 0 as scalar rows
      vec = 1;
    }
    pp->vec = vec;
    pp->rows = total / d[0].size;
    if (text) *text = "permute: row copy, vec=" + std::to_string(vec) + ", nd=" + std::to_string(pp->nd);
  } else {
    pp->mode = 1;
    pp->tdim_in = tin;
    pp->batch = total / (d[0].size * d[tin].size);
    if (text) *text = "permute: 64x64 tile transpose, nd=" + std::to_string(pp->nd);
  }
  return EIR_SUCCESS;
}

// ------------------------------------------------------------- TC lowering
int dim_index_with_unit_stride(std::vector<LDim> const &d, int type, bool left) {
  for (int i = 0; i < (int)d.size(); ++i)
    if (d[i].type == type && (left ? d[i].sl : d[i].sr) == 1) return i;
  return -1;
}

bool try_tc(eir_plan *p, std::string *why) {
  std::vector<LDim> &d = p->dims;
  int kind;
  if (p->dt_l == EIR_BF16 && p->dt_r == EIR_BF16 && p->dt_o == EIR_FP32) {
    if (p->comp != EIR_COMPUTE_DEFAULT && p->comp != EIR_COMPUTE_BF16) {
      *why = "bf16 inputs need BF16/default compute";
      return false;
    }
    kind = 0;
  } else if (p->dt_l == EIR_FP32 && p->dt_r == EIR_FP32 && p->dt_o == EIR_FP32) {
    kind = (p->comp == EIR_COMPUTE_TF32) ? 1 : 2;
  } else if (p->dt_l == EIR_FP64 && p->dt_r == EIR_FP64 && p->dt_o == EIR_FP64) {
    kind = 3;  // FP64 tensor cores (DMMA)
  } else {
    *why = "dtype has no tensor-core path";
    return false;
  }
  const int esize = kind == 0 ? 2 : (kind == 3 ? 8 : 4);
  int nc = 0, nm = 0, nn = 0, nk = 0;
  for (auto const &x : d) {
    if (x.size <= 0 || x.size >= (int64_t(1) << 31)) {
      *why = "dim size out of TMA coordinate range";
      return false;
    }
    if (x.type == EIR_DIM_C) ++nc;
    if (x.type == EIR_DIM_M) ++nm;
    if (x.type == EIR_DIM_N) ++nn;
    if (x.type == EIR_DIM_K) ++nk;
    bool in_l = x.type != EIR_DIM_N, in_r = x.type != EIR_DIM_M, in_o = x.type != EIR_DIM_K;
    if ((in_l && x.sl == 0) || (in_r && x.sr == 0) || (in_o && x.so == 0)) {
      *why = "broadcast (zero-stride) operand dim";
      return false;
    }
  }
  if (nm == 0 || nn == 0 || nk == 0) {
    *why = "needs at least one M, N and K dim";
    return false;
  }
  int64_t cmn = 1, kk = 1;
  for (auto const &x : d) (x.type == EIR_DIM_K ? kk : cmn) *= x.size;
  if (2.0 * (double)cmn * (double)kk < (double)env_int("EIR_TC_MIN_OPS", int64_t(1) << 24)) {
    *why = "below tensor-core size threshold";
    return false;
  }

  int a_k1 = dim_index_with_unit_stride(d, EIR_DIM_K, true);
  int a_m1 = dim_index_with_unit_stride(d, EIR_DIM_M, true);
  int b_k1 = dim_index_with_unit_stride(d, EIR_DIM_K, false);
  int b_n1 = dim_index_with_unit_stride(d, EIR_DIM_N, false);
  bool no_prepack = (p->desc_flags & EIR_FLAG_NO_PREPACK) != 0;

  int kp = -1;
  bool a_mn = false, b_mn = false;
  int prepack = -1;
  auto largest_k = [&]() {
    int best = -1;
    for (int i = 0; i < (int)d.size(); ++i)
      if (d[i].type == EIR_DIM_K && (best < 0 || d[i].size > d[best].size)) best = i;
    return best;
  };
  auto bytes_of = [&](bool left) {
    int64_t n = 1;
    for (auto const &x : d)
      if (x.type == EIR_DIM_C || x.type == EIR_DIM_K || x.type == (left ? EIR_DIM_M : EIR_DIM_N))
        n *= x.size;
    return n * esize;
  };
  if (a_k1 >= 0 && b_k1 >= 0 && a_k1 == b_k1) {
    kp = a_k1;
  } else if (a_k1 >= 0 && b_n1 >= 0) {
    kp = a_k1;
    b_mn = true;
  } else if (a_m1 >= 0 && b_k1 >= 0) {
    kp = b_k1;
    a_mn = true;
  } else if (a_m1 >= 0 && b_n1 >= 0) {
    kp = largest_k();
    a_mn = b_mn = true;
  } else if (!no_prepack && a_k1 >= 0 && b_k1 >= 0) {
    // K-order mismatch: re-layout the smaller operand around the other's K dim
    if (bytes_of(false) <= bytes_of(true)) {
      prepack = 1;
      kp = a_k1;
    } else {
      prepack = 0;
      kp = b_k1;
    }
  } else if (!no_prepack && (a_k1 >= 0 || a_m1 >= 0) && b_k1 < 0 && b_n1 < 0) {
    prepack = 1;
    kp = a_k1 >= 0 ? a_k1 : largest_k();
    a_mn = a_k1 < 0;
  } else if (!no_prepack && (b_k1 >= 0 || b_n1 >= 0) && a_k1 < 0 && a_m1 < 0) {
    prepack = 0;
    kp = b_k1 >= 0 ? b_k1 : largest_k();
    b_mn = b_k1 < 0;
  } else {
    *why = "no unit-stride K or row dim usable for TMA";
    return false;
  }

  // primitive M / N
  int mp = -1, np = -1;
  if (a_mn) {
    mp = a_m1;
  } else {
    for (int i = 0; i < (int)d.size(); ++i)
      if (d[i].type == EIR_DIM_M &&
          (mp < 0 || std::llabs(d[i].so) < std::llabs(d[mp].so) ||
           (std::llabs(d[i].so) == std::llabs(d[mp].so) && d[i].size > d[mp].size)))
        mp = i;
  }
  if (b_mn) {
    np = b_n1;
  } else {
    for (int i = 0; i < (int)d.size(); ++i)
      if (d[i].type == EIR_DIM_N &&
          (np < 0 || d[i].size > d[np].size ||
           (d[i].size == d[np].size && std::llabs(d[i].so) < std::llabs(d[np].so))))
        np = i;
  }

  // Operand copies into the plan's workspace, one per operand at most:
  //  * K-order mismatch (prepack): the operand re-laid out with its dims in
  //    descending stride order except the primitive K dim, which becomes
  //    innermost (the operand is K-major afterwards);
  //  * TF32 compute: each FP32 operand rounded to the nearest TF32 value
  //    (ties to even) while it is copied, dims kept in their order, so the
  //    tensor cores (which ignore the 13 low mantissa bits of an FP32 word)
  //    multiply exactly the TF32-rounded operands of the oracle's model.
  const bool round_tf32 = kind == 1;
  const bool copy_l = prepack == 0 || round_tf32, copy_r = prepack == 1 || round_tf32;
  auto packed_layout = [&](bool left, bool k_inner) {
    std::vector<int64_t> ps(d.size(), 0);
    std::vector<int> ids;
    for (int i = 0; i < (int)d.size(); ++i)
      if (d[i].type == EIR_DIM_C || d[i].type == EIR_DIM_K ||
          d[i].type == (left ? EIR_DIM_M : EIR_DIM_N))
        if (!(k_inner && i == kp)) ids.push_back(i);
    std::stable_sort(ids.begin(), ids.end(), [&](int a, int b) {
      return std::llabs(left ? d[a].sl : d[a].sr) > std::llabs(left ? d[b].sl : d[b].sr);
    });
    if (k_inner) ids.push_back(kp);
    int64_t s = 1;
    for (int j = (int)ids.size() - 1; j >= 0; --j) {
      ps[ids[j]] = s;
      s *= d[ids[j]].size;
    }
    return ps;
  };
  const std::vector<int64_t> packed_l = copy_l ? packed_layout(true, prepack == 0) : std::vector<int64_t>();
  const std::vector<int64_t> packed_r = copy_r ? packed_layout(false, prepack == 1) : std::vector<int64_t>();
  // a re-laid-out operand is K-major now (the kept-order TF32 copy keeps its major-ness)
  if (prepack == 0) a_mn = false;
  if (prepack == 1) b_mn = false;
  auto sl_of = [&](int i) { return copy_l ? packed_l[i] : d[i].sl; };
  auto sr_of = [&](int i) { return copy_r ? packed_r[i] : d[i].sr; };

  // outer K dims and tile loops
  std::vector<int> ko, loops;
  for (int i = 0; i < (int)d.size(); ++i) {
    if (i == kp || i == mp || i == np) continue;
    if (d[i].type == EIR_DIM_K) ko.push_back(i);
    else loops.push_back(i);
  }
  if (ko.size() > 2) {
    *why = "more than two outer K dims";
    return false;
  }
  // the tile loop with the largest output stride becomes the slowest one:
  // tiles then finish slab by slab of the output's outermost dim, which
  // eir_contract_gather moves to the peers one slab at a time
  if (loops.size() > 1) {
    auto outer = std::max_element(loops.begin(), loops.end(), [&](int a, int b) {
      return std::llabs(d[a].so) < std::llabs(d[b].so);
    });
    std::rotate(outer, outer + 1, loops.end());
  }
  if ((int)loops.size() > eir::kMaxTileLoops) {
    *why = "more than four tile-loop dims";
    return false;
  }

  const int bk = eir::tc_block_k(kind);
  // Tile shape. One CTA per 128 x BN tile stages 128 + BN operand rows per K
  // block; a CTA pair (256 x BN over two SMs, kinds BF16 / TF32 / 3xTF32) stages
  // 128 + BN/2 rows per SM for the same 128 x BN outputs per SM. Operand rows
  // staged per SM (the L2 -> SM traffic) set the time of a tile once K is
  // long; minimise waves x (rows per SM + a fixed per-tile overhead).
  int64_t loop_tiles = 1;
  for (int i : loops) loop_tiles *= d[i].size;
  DeviceState *ds = nullptr;
  int num_sms = 148;
  if (device_state(&ds) == EIR_SUCCESS) num_sms = ds->num_sms;
  int bn = 128;
  bool pair = false;
  // Split-K: when one-CTA 128 x 128 tiles would fill under half the SMs and
  // the K walk is long, the K walk is split into slices that run as separate
  // work items (one-CTA kernel; partial tiles reduced by a second kernel)
  int64_t k_blocks_total = ceil_div(d[kp].size, (int64_t)bk);
  for (int i : ko) k_blocks_total *= d[i].size;
  const int64_t tiles_128 = ceil_div(d[mp].size, 128) * ceil_div(d[np].size, 128) * loop_tiles;
  const bool split_k = kind != 3 && env_int("EIR_TC_SPLITK", 1) != 0 && tiles_128 * 2 <= num_sms &&
                       k_blocks_total >= 64;
  if (kind != 3 && !split_k) {
    const int64_t force_bn = env_int("EIR_TC_BN", 0);     // tuning override: 128 or 256
    const int64_t force_pair = env_int("EIR_TC_PAIR", -1);  // tuning override: 0 or 1
    double best = 0.0;
    for (int pr = 0; pr < 2; ++pr) {
      if (force_pair == 0 && pr == 1) continue;
      if (force_pair == 1 && pr == 0 && d[mp].size > 128) continue;
      if (pr == 1 && d[mp].size <= 128) continue;  // a pair tile would be half empty
      for (int cbn : {128, 256}) {
        if (kind == 2 && pr == 0 && cbn == 256) continue;  // one-CTA 3xTF32: BN = 128 only
        if ((force_bn == 128 || force_bn == 256) && cbn != force_bn) continue;
        if (cbn == 256 && d[np].size <= 128 && force_bn != 256) continue;
        const int64_t tiles = ceil_div(d[mp].size, pr ? 256 : 128) * ceil_div(d[np].size, cbn) *
                              loop_tiles;
        const int64_t slots = pr ? std::max(1, num_sms / 2) : num_sms;
        const double cost = (double)ceil_div(tiles, slots) * (128 + (pr ? cbn / 2 : cbn) + 64);
        if (best == 0.0 || cost < best) {
          best = cost;
          bn = cbn;
          pair = pr == 1;
        }
      }
    }
  }
  const int tile_m = pair ? 256 : 128;
  // a 128 x BN tile over tiny primitive M / N dims wastes most of each MMA
  {
    double um = (double)d[mp].size / (double)(ceil_div(d[mp].size, tile_m) * tile_m);
    double un = (double)d[np].size / (double)(ceil_div(d[np].size, bn) * bn);
    char const *v = std::getenv("EIR_TC_MIN_UTIL");
    double min_util = (v != nullptr && *v) ? std::atof(v) : 0.25;
    if (um * un < min_util) {
      *why = "tile utilisation of the primitive M/N dims below threshold";
      return false;
    }
  }

  // TMA maps
  auto fill_map = [&](eir::MapSpec &ms, bool left, bool mn, int rowdim, int rows) -> bool {
    ms.dtype = kind == 0 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
             : kind == 3 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT64 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    // 32-bit MN-major operands: the only tcgen05 layout is 128B swizzle with 32B atoms
    ms.swizzle = (mn && esize == 4) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
    auto st = [&](int i) { return left ? sl_of(i) : sr_of(i); };
    int first = mn ? rowdim : kp, second = mn ? kp : rowdim;
    if (st(first) != 1) return false;
    ms.dims[0] = (uint64_t)d[first].size;
    ms.dims[1] = (uint64_t)d[second].size;
    ms.box[0] = mn ? (uint32_t)(128 / esize) : (uint32_t)bk;
    ms.box[1] = mn ? (uint32_t)bk : (uint32_t)rows;
    int64_t s1 = st(second) * esize;
    if (s1 <= 0 || s1 % 16 != 0 || s1 >= (int64_t(1) << 40)) return false;
    ms.strides_bytes[0] = (uint64_t)s1;
    int8_t *src = left ? p->tcp.a_src : p->tcp.b_src;
    for (int j = 0; j < 5; ++j) src[j] = eir::kSrcNone;
    int slot = 2;
    int64_t maxs = s1;
    for (int j = 0; j < (int)ko.size(); ++j) {
      if (slot > 4) return false;
      int64_t s = st(ko[j]) * esize;
      if (s <= 0 || s % 16 != 0 || s >= (int64_t(1) << 40)) return false;
      ms.dims[slot] = (uint64_t)d[ko[j]].size;
      ms.strides_bytes[slot - 1] = (uint64_t)s;
      src[slot] = (int8_t)(eir::kSrcKo0 + j);
      maxs = std::max(maxs, s);
      ++slot;
    }
    for (int j = 0; j < (int)loops.size(); ++j) {
      int i = loops[j];
      bool has = d[i].type == EIR_DIM_C || d[i].type == (left ? EIR_DIM_M : EIR_DIM_N);
      if (!has) continue;
      if (slot > 4) return false;
      int64_t s = st(i) * esize;
      if (s <= 0 || s % 16 != 0 || s >= (int64_t(1) << 40)) return false;
      ms.dims[slot] = (uint64_t)d[i].size;
      ms.strides_bytes[slot - 1] = (uint64_t)s;
      src[slot] = (int8_t)(eir::kSrcLoop0 + j);
      maxs = std::max(maxs, s);
      ++slot;
    }
    for (; slot < 5; ++slot) {
      ms.dims[slot] = 1;
      ms.strides_bytes[slot - 1] = (uint64_t)maxs;
    }
    return true;
  };
  if (!fill_map(p->map_a, true, a_mn, mp, 128)) {
    *why = "left operand strides not TMA-compatible";
    return false;
  }
  if (!fill_map(p->map_b, false, b_mn, np, pair ? bn / 2 : bn)) {
    *why = "right operand strides not TMA-compatible";
    return false;
  }

  eir::TcParams &t = p->tcp;
  t.m_size = d[mp].size;
  t.n_size = d[np].size;
  t.kp_size = d[kp].size;
  t.so_m = d[mp].so;
  t.so_n = d[np].so;
  t.sa_m = d[mp].sa;
  t.sa_n = d[np].sa;
  t.n_loops = (int)loops.size();
  for (int j = 0; j < eir::kMaxTileLoops; ++j) {
    t.loop_size[j] = j < t.n_loops ? d[loops[j]].size : 1;
    t.loop_so[j] = j < t.n_loops ? d[loops[j]].so : 0;
    t.loop_sa[j] = j < t.n_loops ? d[loops[j]].sa : 0;
  }
  t.ko_size[0] = ko.size() > 0 ? d[ko[0]].size : 1;
  t.ko_size[1] = ko.size() > 1 ? d[ko[1]].size : 1;
  t.m_tiles = (int32_t)ceil_div(t.m_size, tile_m);
  t.n_tiles = (int32_t)ceil_div(t.n_size, bn);
  t.kp_blocks = (int32_t)ceil_div(t.kp_size, bk);
  int64_t ksteps = (int64_t)t.kp_blocks * t.ko_size[0] * t.ko_size[1];
  if (ksteps >= (int64_t(1) << 31)) {
    *why = "K too large";
    return false;
  }
  t.k_steps = (int32_t)ksteps;
  t.total_tiles = (int64_t)t.m_tiles * t.n_tiles;
  for (int j = 0; j < t.n_loops; ++j) t.total_tiles *= t.loop_size[j];
  if (t.total_tiles >= (int64_t(1) << 31)) {  // the kernels index tiles in 32 bits
    *why = "too many output tiles";
    return false;
  }
  t.first_touch = p->first;
  t.last_touch = p->last;
  t.group_m = (int32_t)std::max<int64_t>(1, env_int("EIR_TC_GROUP_M", 16));
  // K blocks per ring stage: two (larger stages) whenever there are at least two K blocks
  const bool ksub_ok = kind == 0 || kind == 1;  // 3xTF32 and FP64 use one K block per stage
  int ksub = (ksub_ok && t.k_steps >= 2) ? 2 : 1;
  int64_t force_ksub = env_int("EIR_TC_KSUB", 0);  // tuning override: 1 or 2
  if (ksub_ok && (force_ksub == 1 || force_ksub == 2)) ksub = (int)force_ksub;
  p->tc_ksub = ksub;
  // split-K slices: enough work items for the SMs, >= 8 stages per slice
  t.base_tiles = t.total_tiles;
  t.split_k = 1;
  t.ws_slice = 0;
  p->split_ws_offset = 0;
  if (split_k) {
    const int64_t n_st = ceil_div((int64_t)t.k_steps, (int64_t)ksub);
    const int64_t s = std::min<int64_t>(std::min<int64_t>(num_sms / t.total_tiles, n_st / 8), 32);
    const int64_t out_elems = t.m_size * t.n_size * loop_tiles;
    if (s >= 2 && s * out_elems * 4 <= (int64_t(1) << 30)) {
      t.split_k = (int32_t)s;
      t.ws_slice = out_elems;
      t.total_tiles *= s;
    }
  }
  // accumulation chunks (the tensor core's FP32 accumulation drifts by about
  // 2e-8 relative per accumulating MMA; every chunk costs the epilogue a
  // read-modify-write of the output tile): 1024 K for 3xTF32 (FP32-exact,
  // three MMAs per 8 K: <= 384 per chunk, <= ~8e-6), 8192 K for TF32 (whose
  // inputs already carry ~1e-3) and for BF16 (<= 1024 / 512 MMAs)
  {
    const int64_t chunk_k = kind == 2 ? 1024 : 8192;
    const int64_t per_stage = (int64_t)bk * ksub;
    const int64_t n_stages = ceil_div((int64_t)t.k_steps, (int64_t)ksub);
    const int64_t kc_max = std::max<int64_t>(1, chunk_k / per_stage);
    // chunks of equal length (a short last chunk would leave its epilogue
    // nothing to overlap with)
    const int64_t n_chunks = ceil_div(n_stages, kc_max);
    t.k_chunk = n_chunks > 1 ? (int32_t)ceil_div(n_stages, n_chunks) : 0;
  }

  p->tc = true;
  p->tc_kind = kind;
  p->tc_bn = bn;
  p->tc_pair = pair;
  p->a_mn = a_mn;
  p->b_mn = b_mn;
  p->tc_esize = esize;
  p->prepack = prepack;

  // the operand copies' permute plans and their places in the workspace
  p->ws_bytes = 0;
  for (int side = 0; side < 2; ++side) {
    const bool left = side == 0;
    if (!(left ? copy_l : copy_r)) continue;
    std::vector<int64_t> const &ps = left ? packed_l : packed_r;
    std::vector<int64_t> sz, si, so;
    for (int i = 0; i < (int)d.size(); ++i)
      if (d[i].type == EIR_DIM_C || d[i].type == EIR_DIM_K ||
          d[i].type == (left ? EIR_DIM_M : EIR_DIM_N)) {
        sz.push_back(d[i].size);
        si.push_back(left ? d[i].sl : d[i].sr);
        so.push_back(ps[i]);
      }
    eir_plan *pre = nullptr;
    int rc = eir_permute_plan_create((int32_t)sz.size(), sz.data(), si.data(), so.data(),
                                     left ? p->dt_l : p->dt_r, &pre);
    if (rc != EIR_SUCCESS) {
      *why = "operand copy planning failed";
      if (p->pre_l) eir_plan_destroy(p->pre_l);
      p->pre_l = nullptr;
      p->tc = false;
      return false;
    }
    pre->perm.round_tf32 = round_tf32 ? 1 : 0;
    (left ? p->pre_l : p->pre_r) = pre;
    (left ? p->ws_off_l : p->ws_off_r) = p->ws_bytes;
    p->ws_bytes = (p->ws_bytes + bytes_of(left) + 255) / 256 * 256;
  }
  if (t.split_k > 1) {
    p->split_ws_offset = p->ws_bytes;
    p->ws_bytes = p->split_ws_offset + (int64_t)t.split_k * t.ws_slice * 4;
  }

  char buf[512];
  std::snprintf(buf, sizeof(buf),
                "tc kind=%s %sBN=%d KSUB=%d A=%s B=%s M=%lld N=%lld Kp=%lld ko=%lldx%lld loops=%d "
                "tiles=%lld ksteps=%d prepack=%s splitk=%d%s",
                kind == 0 ? "bf16" : kind == 1 ? "tf32" : kind == 2 ? "3xtf32" : "fp64-dmma",
                pair ? "pair BM=256 " : "", bn,
                p->tc_ksub, a_mn ? "MN" : "K",
                b_mn ? "MN" : "K", (long long)t.m_size, (long long)t.n_size, (long long)t.kp_size,
                (long long)t.ko_size[0], (long long)t.ko_size[1], t.n_loops,
                (long long)t.total_tiles, t.k_steps,
                prepack < 0 ? "none" : (prepack == 0 ? "left" : "right"), (int)t.split_k,
                round_tf32 ? " tf32-rounded-copies" : "");
  *why = buf;
  return true;
}

bool valid_first(int k) {
  return k == EIR_KTYPE_ZERO || k == EIR_KTYPE_COPY || k == EIR_KTYPE_ADD || k == EIR_KTYPE_UNDEFINED;
}
bool valid_last(int k) {
  return k == EIR_KTYPE_RELU || k == EIR_KTYPE_ADD || k == EIR_KTYPE_UNDEFINED;
}

// Output layout facts for eir_contract_gather: whether the output is one
// contiguous block, and its slabs along the outermost output dim when that
// dim is the tensor-core kernel's slowest tile loop (tiles finish slab by slab).
void plan_gather(eir_plan *p) {
  std::vector<LDim> od;
  for (auto const &x : p->dims)
    if (x.type != EIR_DIM_K) od.push_back(x);
  std::sort(od.begin(), od.end(), [](LDim const &a, LDim const &b) { return a.so < b.so; });
  bool dense = true;
  int64_t elems = 1;
  for (auto const &x : od) {
    if (x.so != elems) dense = false;
    elems *= x.size;
  }
  p->out_dense = dense;
  p->out_elems = elems;
  p->slab_count = 1;
  p->slab_elems = elems;
  p->slab_loop = -1;
  p->slab_counted = false;
  p->slab_target = 1;
  eir::TcParams const &t = p->tcp;
  const bool tc = p->family == EIR_FAMILY_TC || p->family == EIR_FAMILY_DMMA;
  if (!dense || !tc || t.split_k > 1 || t.n_loops < 1 || od.empty()) return;
  const int j = t.n_loops - 1;
  if (t.loop_so[j] != od.back().so || t.loop_size[j] != od.back().size || t.loop_size[j] < 2) return;
  p->slab_count = t.loop_size[j];
  p->slab_elems = t.loop_so[j];
  p->slab_loop = j;
  if (p->family == EIR_FAMILY_DMMA) {
    // every math warp of the DMMA kernel counts each tile it stores
    p->slab_counted = true;
    p->slab_target = (uint32_t)(t.total_tiles / p->slab_count) * 8u;
  }
}

// events around a plan's main kernel when profiling is enabled
struct ProfScope {
  eir_plan *p;
  cudaStream_t st;
  cudaEvent_t e1 = nullptr;
  ProfScope(eir_plan *plan, cudaStream_t s) : p(plan), st(s) {
    if (!p->profile) return;
    if (p->prof_used == p->prof_events.size()) {
      cudaEvent_t a, b;
      if (cudaEventCreate(&a) != cudaSuccess) return;
      if (cudaEventCreate(&b) != cudaSuccess) {
        cudaEventDestroy(a);
        return;
      }
      p->prof_events.emplace_back(a, b);
    }
    cudaEventRecord(p->prof_events[p->prof_used].first, st);
    e1 = p->prof_events[p->prof_used].second;
  }
  ~ProfScope() {
    if (e1 == nullptr) return;
    cudaEventRecord(e1, st);
    p->prof_used++;
  }
};

int run_simt(eir_plan *p, void const *l, void const *r, void const *aux, void *out,
             eir::PeerOutputs const *peers, cudaStream_t st) {
  ProfScope prof(p, st);
  cudaError_t e;
  if (p->simt_direct) {
    eir::DirectParams dp = p->direct;
    if (peers != nullptr) dp.peers = *peers;
    e = eir::launch_simt_direct(p->dt_l, p->dt_r, p->dt_o, dp, l, r, aux, out, st);
  } else {
    eir::SimtParams sp = p->simt;
    if (peers != nullptr) sp.peers = *peers;
    e = eir::launch_simt_contract(p->dt_l, p->dt_r, p->dt_o, sp, l, r, aux, out, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "simt contraction launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return EIR_SUCCESS;
}

}  // namespace

// library-internal helpers shared with other translation units (eir_plan.h)
namespace eir {
int api_set_error(int code, char const *msg) { return set_error(code, msg); }
int api_cuda_fail(cudaError_t e, char const *where) { return cuda_fail(e, where); }
int api_encode_map(MapSpec const &s, void const *ptr, CUtensorMap *m) { return encode_map(s, ptr, m); }
void api_count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
int api_launch_tc_split(eir_plan const *p, CUtensorMap const &ma, CUtensorMap const &mb,
                        TcParams const &tp, void const *aux, void *out, float *ws, int num_sms,
                        cudaStream_t st) {
  // the slices write dense partial tiles [slice][tile loops][n][m] with a
  // ZERO first touch and no last touch; the reduction applies the plan's
  TcParams ts = tp;
  ts.first_touch = 0;
  ts.last_touch = 99;
  ts.so_m = 1;
  ts.so_n = tp.m_size;
  ts.sa_m = ts.sa_n = 0;
  int64_t stride = tp.m_size * tp.n_size;
  for (int i = 0; i < kMaxTileLoops; ++i) {
    ts.loop_so[i] = stride;
    ts.loop_sa[i] = 0;
    if (i < tp.n_loops) stride *= tp.loop_size[i];
  }
  ts.peers = PeerOutputs();
  cudaError_t e = api_launch_tc(p, ma, mb, ts, nullptr, ws, num_sms, st);
  if (e != cudaSuccess) return cuda_fail(e, "tc split-K launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  e = launch_splitk_reduce(tp, ws, static_cast<float const *>(aux), static_cast<float *>(out), num_sms, st);
  if (e != cudaSuccess) return cuda_fail(e, "split-K reduction launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return EIR_SUCCESS;
}
cudaError_t api_launch_tc(eir_plan const *p, CUtensorMap const &ma, CUtensorMap const &mb,
                          TcParams const &tp, void const *aux, void *out, int num_sms,
                          cudaStream_t st) {
  if (p->tc_kind == 3)
    return launch_dmma_contract(p->a_mn, p->b_mn, ma, mb, tp, static_cast<double const *>(aux),
                                static_cast<double *>(out), num_sms, st);
  if (p->tc_pair)
    return launch_tc_pair_contract(p->tc_kind, p->tc_bn, p->tc_ksub, p->a_mn, p->b_mn, ma, mb, tp,
                                   static_cast<float const *>(aux), static_cast<float *>(out), st);
  return launch_tc_contract(p->tc_kind, p->tc_bn, p->tc_ksub, p->a_mn, p->b_mn, ma, mb, tp,
                            static_cast<float const *>(aux), static_cast<float *>(out), num_sms, st);
}
}  // namespace eir

// =================================================================== C-ABI
extern "C" {

int eir_version(void) { return 1; }

char const *eir_last_error_string(void) { return g_last_error.c_str(); }

int64_t eir_launch_count(void) { return g_launches.load(); }

// Complex contraction (one EIR_DIM_CPX dim of size 2 in left, right and out,
// CPX_MADD main kernel; reference: BinaryContraction.cpp:453-462 for num_ops,
// ContractionBackend.cpp:663-675 for the complex strides). Lowered to one real
// contraction: out[co] = sum_ci A[ci] * B'[ci][co] with B' = [[Br, Bi], [-Bi, Br]],
// i.e. the complex dim becomes a K dim of A (ci) and an N dim of out (co),
// and B' is the right operand expanded into four packed real blocks.
static int create_complex_plan(eir_contract_desc const *desc, eir_plan **plan_out) {
  int cpx = -1;
  for (int i = 0; i < desc->num_dims; ++i) {
    if (desc->dims[i].type != EIR_DIM_CPX) continue;
    if (cpx >= 0) return set_error(EIR_INVALID_CPX_DIM, "more than one complex dim");
    cpx = i;
  }
  eir_dim const &x = desc->dims[cpx];
  if (x.size != 2) return set_error(EIR_INVALID_CPX_DIM, "the complex dim must have size 2");
  if (desc->ktype_main != EIR_KTYPE_CPX_MADD ||
      (desc->ktype_first_touch != EIR_KTYPE_CPX_ZERO && desc->ktype_first_touch != EIR_KTYPE_UNDEFINED) ||
      desc->ktype_last_touch != EIR_KTYPE_UNDEFINED)
    return set_error(EIR_INVALID_KTYPE, "complex contractions take CPX_ZERO / CPX_MADD only");
  const int dt = desc->dtype_left;
  if (dt != desc->dtype_right || dt != desc->dtype_out || (dt != EIR_FP32 && dt != EIR_FP64))
    return set_error(EIR_INVALID_DTYPE, "complex contractions: FP32 or FP64 throughout");
  // B's other dims, packed with the smallest right stride innermost
  std::vector<int> bdims;
  for (int i = 0; i < desc->num_dims; ++i) {
    int t = desc->dims[i].type;
    if (i != cpx && (t == EIR_DIM_C || t == EIR_DIM_N || t == EIR_DIM_K)) bdims.push_back(i);
  }
  if ((int)bdims.size() > eir::kMaxPermDims)
    return set_error(EIR_COMPILATION_FAILED, "too many dims in the right operand");
  std::stable_sort(bdims.begin(), bdims.end(), [&](int a, int b) {
    return std::llabs(desc->dims[a].stride_right) < std::llabs(desc->dims[b].stride_right);
  });
  std::vector<int64_t> packed(desc->num_dims, 0);
  int64_t nb = 1;
  for (int i : bdims) {
    packed[i] = nb;
    nb *= desc->dims[i].size;
  }
  // the real problem
  std::vector<eir_dim> dims;
  for (int i = 0; i < desc->num_dims; ++i) {
    if (i == cpx) continue;
    eir_dim y = desc->dims[i];
    y.stride_right = packed[i];
    dims.push_back(y);
  }
  eir_dim ci{}, co{};
  ci.type = EIR_DIM_K;
  ci.size = 2;
  ci.stride_left = x.stride_left;
  ci.stride_right = 2 * nb;
  co.type = EIR_DIM_N;
  co.size = 2;
  co.stride_right = nb;
  co.stride_out = x.stride_out;
  dims.push_back(ci);
  dims.push_back(co);
  eir_contract_desc rd = *desc;
  rd.num_dims = (int32_t)dims.size();
  rd.dims = dims.data();
  rd.ktype_first_touch = desc->ktype_first_touch == EIR_KTYPE_CPX_ZERO ? EIR_KTYPE_ZERO : EIR_KTYPE_UNDEFINED;
  rd.ktype_main = EIR_KTYPE_MADD;
  eir_plan *inner = nullptr;
  int rc = eir_contract_plan_create(&rd, &inner);
  if (rc != EIR_SUCCESS) return rc;

  eir_plan *p = new eir_plan();
  p->what = 1;
  p->dt_l = p->dt_r = p->dt_o = dt;
  p->comp = desc->dtype_comp;
  p->first = desc->ktype_first_touch;
  p->last = desc->ktype_last_touch;
  p->desc_flags = desc->flags;
  p->family = inner->family;
  p->num_ops = inner->num_ops;  // 8|C||M||N||K| - 2|C||M||N| with ZERO: the reference's count
  p->empty = inner->empty;
  p->cpx_inner = inner;
  p->esize = dt == EIR_FP64 ? 8 : 4;
  p->cpx_stride_right = x.stride_right;
  eir::PermuteParams &e = p->cpx_expand;
  e = eir::PermuteParams();
  e.nd = (int32_t)bdims.size();
  for (int j = 0; j < e.nd; ++j) {
    e.size[j] = desc->dims[bdims[j]].size;
    e.sin[j] = desc->dims[bdims[j]].stride_right;
    e.sout[j] = packed[bdims[j]];
  }
  e.total = nb;
  p->ws_bytes = 4 * nb * p->esize;
  p->text = "complex: right operand expanded to [[Br, Bi], [-Bi, Br]] (" + std::to_string(nb) +
            " x 4 elements) + " + inner->text;
  *plan_out = p;
  return EIR_SUCCESS;
}

int eir_contract_plan_create(eir_contract_desc const *desc, eir_plan **plan_out) {
  if (desc == nullptr || plan_out == nullptr)
    return set_error(EIR_INVALID_ARGUMENT, "null descriptor or plan pointer");
  *plan_out = nullptr;
  if (desc->num_dims < 0 || (desc->num_dims > 0 && desc->dims == nullptr))
    return set_error(EIR_INVALID_ARGUMENT, "bad dims");
  for (int i = 0; i < desc->num_dims; ++i)
    if (desc->dims[i].type == EIR_DIM_CPX) return create_complex_plan(desc, plan_out);
  const int dl = desc->dtype_left, dr = desc->dtype_right, dout = desc->dtype_out;
  bool dt_ok = (dout == EIR_FP64 && dl == EIR_FP64 && dr == EIR_FP64) ||
               (dout == EIR_FP32 && (dl == EIR_FP32 || dl == EIR_BF16) &&
                (dr == EIR_FP32 || dr == EIR_BF16));
  if (!dt_ok) return set_error(EIR_INVALID_DTYPE, "unsupported dtype combination");
  if (desc->dtype_comp < EIR_COMPUTE_DEFAULT || desc->dtype_comp > EIR_COMPUTE_BF16)
    return set_error(EIR_INVALID_DTYPE, "unsupported compute type");
  if (dout == EIR_FP64 && desc->dtype_comp != EIR_COMPUTE_DEFAULT && desc->dtype_comp != EIR_COMPUTE_FP64)
    return set_error(EIR_INVALID_DTYPE, "FP64 data needs FP64 compute");
  if (!valid_first(desc->ktype_first_touch) || desc->ktype_main != EIR_KTYPE_MADD ||
      !valid_last(desc->ktype_last_touch))
    return set_error(EIR_INVALID_KTYPE, "unsupported kernel type");
  bool uses_aux = desc->ktype_first_touch == EIR_KTYPE_COPY || desc->ktype_first_touch == EIR_KTYPE_ADD ||
                  desc->ktype_last_touch == EIR_KTYPE_ADD;

  eir_plan *p = new eir_plan();
  p->what = 1;
  p->dt_l = dl;
  p->dt_r = dr;
  p->dt_o = dout;
  p->comp = desc->dtype_comp;
  p->first = desc->ktype_first_touch;
  p->last = desc->ktype_last_touch;
  p->desc_flags = desc->flags;

  std::vector<LDim> dims;
  int64_t sc = 1, sm = 1, sn = 1, sk = 1;
  for (int i = 0; i < desc->num_dims; ++i) {
    eir_dim const &x = desc->dims[i];
    if (x.type < EIR_DIM_C || x.type > EIR_DIM_K || x.size < 0) {
      delete p;
      return set_error(EIR_INVALID_ARGUMENT, "bad dim type or size");
    }
    LDim y;
    y.type = x.type;
    y.size = x.size;
    y.sl = (x.type == EIR_DIM_N) ? 0 : x.stride_left;
    y.sr = (x.type == EIR_DIM_M) ? 0 : x.stride_right;
    y.so = (x.type == EIR_DIM_K) ? 0 : x.stride_out;
    y.sa = (x.type == EIR_DIM_K || !uses_aux) ? 0 : x.stride_out_aux;
    if (x.size == 0 && x.type != EIR_DIM_K) p->empty = true;
    (x.type == EIR_DIM_C ? sc : x.type == EIR_DIM_M ? sm : x.type == EIR_DIM_N ? sn : sk) *= x.size;
    dims.push_back(y);
  }
  p->num_ops = 2 * sc * sm * sn * sk;
  if (p->first == EIR_KTYPE_ZERO) p->num_ops -= sc * sm * sn;

  // Operand roles (the reference's swap_inputs rule, BinaryPrimitives.cpp:87-134):
  // the output's unit-stride dim should be an M dim. The tensor-core epilogues
  // hold one output row per thread (TMEM lane) and store a column of 32 rows
  // per warp instruction, which coalesces only along M; with the output
  // contiguous along N every lane would write its own row segment. So when the
  // output's fastest dim is an N dim, left and right change roles (M <-> N);
  // the products, hence the result, are the same.
  {
    int fastest = -1;
    for (int i = 0; i < (int)dims.size(); ++i)
      if (dims[i].type != EIR_DIM_K && dims[i].size > 1 && dims[i].so != 0 &&
          (fastest < 0 || std::llabs(dims[i].so) < std::llabs(dims[fastest].so)))
        fastest = i;
    if (fastest >= 0 && dims[fastest].type == EIR_DIM_N && sm > 1) {
      p->swapped = true;
      for (auto &x : dims) {
        if (x.type == EIR_DIM_M) x.type = EIR_DIM_N;
        else if (x.type == EIR_DIM_N) x.type = EIR_DIM_M;
        std::swap(x.sl, x.sr);
      }
      std::swap(p->dt_l, p->dt_r);
    }
  }

  p->dims = simplify_dims(dims);
  for (int ty = EIR_DIM_C; ty <= EIR_DIM_K; ++ty) {
    eir::GroupDims *g = ty == EIR_DIM_C ? &p->simt.c : ty == EIR_DIM_M ? &p->simt.m
                      : ty == EIR_DIM_N ? &p->simt.n : &p->simt.k;
    if (build_group(p->dims, ty, g) != 0) {
      delete p;
      return set_error(EIR_COMPILATION_FAILED, "too many non-fusable dims of one type");
    }
  }
  p->simt.first_touch = p->first;
  p->simt.last_touch = p->last;
  p->simt.round_tf32 = (p->comp == EIR_COMPUTE_TF32 && dl == EIR_FP32 && dr == EIR_FP32) ? 1 : 0;
  p->simt.a_kfast = min_abs_stride(p->dims, EIR_DIM_K, true) < min_abs_stride(p->dims, EIR_DIM_M, true);
  p->simt.b_kfast = min_abs_stride(p->dims, EIR_DIM_K, false) < min_abs_stride(p->dims, EIR_DIM_N, false);
  p->simt.m_tiles = ceil_div(p->simt.m.total, 64);
  p->simt.n_tiles = ceil_div(p->simt.n.total, 64);
  build_direct(p);

  std::string why = "forced";
  if (!p->empty && !(desc->flags & EIR_FLAG_FORCE_SIMT) && try_tc(p, &why)) {
    p->family = p->tc_kind == 3 ? EIR_FAMILY_DMMA : EIR_FAMILY_TC;
  } else {
    p->family = EIR_FAMILY_SIMT;
  }
  plan_gather(p);
  std::string dims_txt;
  for (auto const &x : p->dims) {
    dims_txt += type_name(x.type);
    dims_txt += std::to_string(x.size) + " ";
  }
  const bool tensor_cores = p->family == EIR_FAMILY_TC || p->family == EIR_FAMILY_DMMA;
  p->text = (tensor_cores ? why : "simt (" + why + (p->simt_direct ? "; one output per thread" : "") + ")") +
            " | dims: " + dims_txt;
  if (p->swapped) p->text += "| operands swapped (output contiguous along the right operand) ";
  if (p->out_dense)
    p->text += "| gather: " + std::to_string(p->slab_count) + " slab(s)" +
               (p->slab_counted ? ", counted by the kernel" : ", released after the kernel");
  *plan_out = p;
  return EIR_SUCCESS;
}

}  // extern "C"

namespace {

// one launch of a permute plan (no device-state lookup, nothing allocated)
int run_permute(eir_plan *p, void const *in, void *out, int num_sms, cudaStream_t st) {
  eir::PermuteParams pp = p->perm;
  if (pp.mode == 0 && pp.vec > 1 &&
      ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) % (pp.vec * p->esize)))
    pp.vec = 1;
  ProfScope prof(p, st);
  cudaError_t e = eir::launch_permute(p->esize, pp, in, out, num_sms, st, p->unary_zero);
  if (e != cudaSuccess) return cuda_fail(e, "permute launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return EIR_SUCCESS;
}

bool takes_tensor_cores(eir_plan const *p, void const *l, void const *r) {
  // TMA needs 16-byte aligned bases; otherwise the generic path reads the operands
  return (p->family == EIR_FAMILY_TC || p->family == EIR_FAMILY_DMMA) &&
         !((reinterpret_cast<uintptr_t>(l) | reinterpret_cast<uintptr_t>(r)) & 15);
}

// eir_contract and its variants (eir::api_contract): peer outputs
// (eir_contract_peers), slab counters (eir_contract_gather), and a caller's
// workspace, error word and SM count (eir_contract_no_alloc, which must not
// reach an allocation: ws_ext / err_ext non-null)
int contract_impl(eir_plan *p, void const *l, void const *r, void const *aux, void *out,
                  eir::PeerOutputs const *peers, void *stream, uint32_t *slab_ctr = nullptr,
                  void *ws_ext = nullptr, uint32_t *err_ext = nullptr, int num_sms_ext = 0) {
  if (p == nullptr || p->what != 1) return set_error(EIR_INVALID_ARGUMENT, "not a contraction plan");
  if (p->empty) return EIR_SUCCESS;
  if (l == nullptr || r == nullptr || out == nullptr)
    return set_error(EIR_NO_DATA_PTR_PROVIDED, "null operand pointer");
  bool uses_aux = p->first == EIR_KTYPE_COPY || p->first == EIR_KTYPE_ADD || p->last == EIR_KTYPE_ADD;
  if (uses_aux && aux == nullptr) return set_error(EIR_NO_DATA_PTR_PROVIDED, "null aux pointer");
  if (p->swapped) std::swap(l, r);  // the plan's left operand is the caller's right one
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p->cpx_inner != nullptr) {
    if (ws_ext != nullptr) return set_error(EIR_INVALID_ARGUMENT, "complex plans need their own workspace");
    // complex: expand the right operand into the workspace, then the real plan
    int dev = 0;
    cudaGetDevice(&dev);
    if (p->ws == nullptr || p->ws_device != dev) {
      if (p->ws != nullptr) cudaFree(p->ws);
      cudaError_t e = cudaMalloc(&p->ws, (size_t)std::max<int64_t>(p->ws_bytes, 16));
      if (e != cudaSuccess) {
        p->ws = nullptr;
        return cuda_fail(e, "cudaMalloc(workspace)");
      }
      p->ws_device = dev;
    }
    DeviceState *ds = nullptr;
    int rc = device_state(&ds);
    if (rc != EIR_SUCCESS) return rc;
    cudaError_t e = eir::launch_cpx_expand(p->esize, p->cpx_expand, p->cpx_stride_right, r, p->ws,
                                           ds->num_sms, st);
    if (e != cudaSuccess) return cuda_fail(e, "complex expansion launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return contract_impl(p->cpx_inner, l, p->ws, aux, out, peers, stream);
  }
  if (!takes_tensor_cores(p, l, r)) return run_simt(p, l, r, aux, out, peers, st);

  uint32_t *err = err_ext;
  int num_sms = num_sms_ext;
  if (err == nullptr) {
    DeviceState *ds = nullptr;
    int rc = device_state(&ds);
    if (rc != EIR_SUCCESS) return rc;
    err = ds->err;
    num_sms = ds->num_sms;
  }
  char *ws = static_cast<char *>(ws_ext);
  if (p->ws_bytes > 0 && ws == nullptr) {  // operand copies and / or split-K partial tiles
    int dev = 0;
    cudaGetDevice(&dev);
    if (p->ws == nullptr || p->ws_device != dev) {
      if (p->ws != nullptr) cudaFree(p->ws);
      cudaError_t e = cudaMalloc(&p->ws, (size_t)p->ws_bytes);
      if (e != cudaSuccess) {
        p->ws = nullptr;
        return cuda_fail(e, "cudaMalloc(workspace)");
      }
      p->ws_device = dev;
    }
    ws = static_cast<char *>(p->ws);
  }
  void const *a_ptr = l, *b_ptr = r;
  int rc = EIR_SUCCESS;
  if (p->pre_l != nullptr) {
    rc = run_permute(p->pre_l, l, ws + p->ws_off_l, num_sms, st);
    if (rc != EIR_SUCCESS) return rc;
    a_ptr = ws + p->ws_off_l;
  }
  if (p->pre_r != nullptr) {
    rc = run_permute(p->pre_r, r, ws + p->ws_off_r, num_sms, st);
    if (rc != EIR_SUCCESS) return rc;
    b_ptr = ws + p->ws_off_r;
  }

  CUtensorMap ma, mb;
  {
    std::lock_guard<std::mutex> lk(p->mu);
    if (p->cache_a.ptr != a_ptr) {
      rc = encode_map(p->map_a, a_ptr, &p->cache_a.map);
      if (rc != EIR_SUCCESS) {
        p->cache_a.ptr = nullptr;
        return rc;
      }
      p->cache_a.ptr = a_ptr;
    }
    if (p->cache_b.ptr != b_ptr) {
      rc = encode_map(p->map_b, b_ptr, &p->cache_b.map);
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
  tp.err = err;
  if (peers != nullptr) tp.peers = *peers;
  if (slab_ctr != nullptr && p->slab_counted) {
    tp.slab_ctr = slab_ctr;
    tp.slab_loop = p->slab_loop;
  }
  ProfScope prof(p, st);
  if (tp.split_k > 1) {
    float *part = reinterpret_cast<float *>(ws + p->split_ws_offset);
    return eir::api_launch_tc_split(p, ma, mb, tp, aux, out, part, num_sms, st);
  }
  cudaError_t e = eir::api_launch_tc(p, ma, mb, tp, aux, out, num_sms, st);
  if (e != cudaSuccess) return cuda_fail(e, "tc contraction launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return EIR_SUCCESS;
}

// cuStreamWaitValue32 through the runtime's driver entry-point query (null
// when the driver does not offer it)
typedef CUresult (*PfnStreamWaitValue32)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
PfnStreamWaitValue32 stream_wait_value32() {
  static PfnStreamWaitValue32 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWaitValue32", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PfnStreamWaitValue32>(f);
  });
  return fn;
}

// frees a plan's gather resources (on the device they were made on)
void release_gather(eir_plan *p) {
  int cur = -1;
  const bool other = p->gather_device >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != p->gather_device;
  if (other) cudaSetDevice(p->gather_device);
  if (p->slab_ctr) cudaFree(p->slab_ctr);
  if (p->gather_start) cudaEventDestroy(p->gather_start);
  for (int i = 0; i < eir::kMaxPeers; ++i) {
    if (p->gather_streams[i]) cudaStreamDestroy(p->gather_streams[i]);
    if (p->gather_done[i]) cudaEventDestroy(p->gather_done[i]);
    p->gather_streams[i] = nullptr;
    p->gather_done[i] = nullptr;
  }
  if (other) cudaSetDevice(cur);
  p->slab_ctr = nullptr;
  p->gather_start = nullptr;
  p->gather_device = -1;
}

// base address of the device allocation holding `ptr` (driver API through
// the runtime's entry-point query, as for the tensor-map encoder)
typedef CUresult (*PfnMemGetAddressRange)(CUdeviceptr *, size_t *, CUdeviceptr);
int allocation_base(void const *ptr, char **base) {
  static PfnMemGetAddressRange fn = nullptr;
  if (fn == nullptr) {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PfnMemGetAddressRange>(f);
  }
  if (fn == nullptr) return set_error(EIR_CUDA_ERROR, "cuMemGetAddressRange unavailable");
  CUdeviceptr b = 0;
  size_t size = 0;
  CUresult r = fn(&b, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return set_error(EIR_CUDA_ERROR, "cuMemGetAddressRange failed (" + std::to_string((int)r) + ")");
  *base = reinterpret_cast<char *>(b);
  return EIR_SUCCESS;
}

}  // namespace

namespace eir {
int api_contract(eir_plan *p, void const *l, void const *r, void const *aux, void *out,
                 PeerOutputs const *peers, void *stream, uint32_t *slab_ctr, void *ws, uint32_t *err,
                 int num_sms) {
  return contract_impl(p, l, r, aux, out, peers, stream, slab_ctr, ws, err, num_sms);
}
int64_t api_workspace_needed(eir_plan const *p, void const *l, void const *r) {
  return takes_tensor_cores(p, l, r) ? p->ws_bytes : 0;
}
}  // namespace eir

extern "C" {

int eir_contract(eir_plan *p, void const *l, void const *r, void const *aux, void *out, void *stream) {
  return contract_impl(p, l, r, aux, out, nullptr, stream);
}

int eir_contract_peers(eir_plan *p, void const *l, void const *r, void const *aux, void *out,
                       int32_t num_peers, void *const *peer_outs, void *stream) {
  if (num_peers < 0 || num_peers > eir::kMaxPeers)
    return set_error(EIR_INVALID_ARGUMENT, "num_peers must be 0.." + std::to_string(eir::kMaxPeers));
  if (num_peers > 0 && peer_outs == nullptr) return set_error(EIR_NO_DATA_PTR_PROVIDED, "null peer list");
  if (p != nullptr && p->what == 1 && p->cpx_inner != nullptr && num_peers > 0)
    return set_error(EIR_INVALID_ARGUMENT, "peer outputs are not supported for complex plans");
  eir::PeerOutputs peers;
  peers.n = num_peers;
  for (int i = 0; i < num_peers; ++i) {
    if (peer_outs[i] == nullptr) return set_error(EIR_NO_DATA_PTR_PROVIDED, "null peer output");
    peers.ptr[i] = peer_outs[i];
  }
  return contract_impl(p, l, r, aux, out, num_peers > 0 ? &peers : nullptr, stream);
}

int eir_contract_gather(eir_plan *p, void const *l, void const *r, void const *aux, void *out,
                        int32_t num_peers, void *const *peer_outs, void *stream) {
  if (num_peers < 0 || num_peers > eir::kMaxPeers)
    return set_error(EIR_INVALID_ARGUMENT, "num_peers must be 0.." + std::to_string(eir::kMaxPeers));
  if (num_peers > 0 && peer_outs == nullptr) return set_error(EIR_NO_DATA_PTR_PROVIDED, "null peer list");
  if (p == nullptr || p->what != 1) return set_error(EIR_INVALID_ARGUMENT, "not a contraction plan");
  if (num_peers == 0 || p->empty) return contract_impl(p, l, r, aux, out, nullptr, stream);
  if (p->cpx_inner != nullptr || !p->out_dense)
    return set_error(EIR_INVALID_ARGUMENT, "eir_contract_gather needs a real plan with a contiguous output");
  for (int i = 0; i < num_peers; ++i)
    if (peer_outs[i] == nullptr) return set_error(EIR_NO_DATA_PTR_PROVIDED, "null peer output");
  if (out == nullptr) return set_error(EIR_NO_DATA_PTR_PROVIDED, "null operand pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t esize = p->dt_o == EIR_FP64 ? 8 : 4;
  const int32_t nslab = (int32_t)p->slab_count;

  // per-plan resources on the current device: slab counters, one copy
  // stream per peer, events joining the copy streams to `stream`
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (p->gather_device != dev) {
    release_gather(p);
    e = cudaMalloc(&p->slab_ctr, sizeof(uint32_t) * (size_t)std::max<int64_t>(nslab, 1));
    if (e != cudaSuccess) {
      p->slab_ctr = nullptr;
      return cuda_fail(e, "cudaMalloc(slab counters)");
    }
    p->gather_device = dev;
    e = cudaEventCreateWithFlags(&p->gather_start, cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
  }
  for (int i = 0; i < num_peers; ++i) {
    if (p->gather_streams[i] == nullptr) {
      e = cudaStreamCreateWithFlags(&p->gather_streams[i], cudaStreamNonBlocking);
      if (e != cudaSuccess) return cuda_fail(e, "cudaStreamCreate(copy stream)");
      e = cudaEventCreateWithFlags(&p->gather_done[i], cudaEventDisableTiming);
      if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
    }
  }

  // 1. counters to zero; the copy streams start after that point of `stream`
  e = cudaMemsetAsync(p->slab_ctr, 0, sizeof(uint32_t) * (size_t)nslab, st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(slab counters)");
  e = cudaEventRecord(p->gather_start, st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  for (int i = 0; i < num_peers; ++i) {
    e = cudaStreamWaitEvent(p->gather_streams[i], p->gather_start, 0);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent");
  }
  // 2. the contraction; a counting kernel moves slab s's counter to
  //    slab_target once all of its tiles are stored
  int rc = contract_impl(p, l, r, aux, out, nullptr, stream, p->slab_ctr);
  if (rc != EIR_SUCCESS) return rc;
  // 3. every counter to its final value once the kernel has completed, so
  //    that no copy below can wait longer than the kernel runs
  e = eir::launch_slab_release(p->slab_ctr, nslab, p->slab_target, st);
  if (e != cudaSuccess) return cuda_fail(e, "slab release launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  // 4. per peer, slab by slab: wait for the slab's count, then copy it
  PfnStreamWaitValue32 wait32 = stream_wait_value32();
  cudaEvent_t kernel_done = nullptr;
  if (wait32 == nullptr) {  // no stream memory operations: copy after the kernel
    kernel_done = p->gather_start;
    e = cudaEventRecord(kernel_done, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  }
  const size_t slab_bytes = (size_t)(p->slab_elems * esize);
  for (int i = 0; i < num_peers; ++i) {
    cudaStream_t cs = p->gather_streams[i];
    if (kernel_done != nullptr) {
      e = cudaStreamWaitEvent(cs, kernel_done, 0);
      if (e != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent");
    }
    for (int32_t sl = 0; sl < nslab; ++sl) {
      const size_t off = (size_t)sl * slab_bytes;
      if (kernel_done == nullptr) {
        CUresult cr = wait32(reinterpret_cast<CUstream>(cs),
                             reinterpret_cast<CUdeviceptr>(p->slab_ctr + sl), p->slab_target,
                             CU_STREAM_WAIT_VALUE_GEQ);
        if (cr != CUDA_SUCCESS)
          return set_error(EIR_CUDA_ERROR, "cuStreamWaitValue32 failed (" + std::to_string((int)cr) + ")");
      }
      e = cudaMemcpyAsync(static_cast<char *>(peer_outs[i]) + off, static_cast<char const *>(out) + off,
                          slab_bytes, cudaMemcpyDeviceToDevice, cs);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(peer slab)");
    }
    // 5. `stream` continues once this peer's copies are done
    e = cudaEventRecord(p->gather_done[i], cs);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    e = cudaStreamWaitEvent(st, p->gather_done[i], 0);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent");
  }
  return EIR_SUCCESS;
}

int eir_copy_to_peers(void const *src, int32_t num_peers, void *const *dsts, int64_t bytes, void *stream) {
  if (bytes < 0 || num_peers < 0 || (num_peers > 0 && (src == nullptr || dsts == nullptr)))
    return set_error(EIR_INVALID_ARGUMENT, "bad argument");
  for (int i = 0; i < num_peers; ++i) {
    if (dsts[i] == nullptr) return set_error(EIR_NO_DATA_PTR_PROVIDED, "null peer destination");
    // one copy per destination; the copy engines move it, no SM is used
    cudaError_t e = cudaMemcpyAsync(dsts[i], src, (size_t)bytes, cudaMemcpyDeviceToDevice,
                                    static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(peer)");
  }
  return EIR_SUCCESS;
}

int eir_ipc_get_handle(void const *dev_ptr, void *handle, int64_t *offset) {
  if (dev_ptr == nullptr || handle == nullptr || offset == nullptr)
    return set_error(EIR_INVALID_ARGUMENT, "null argument");
  char *base = nullptr;
  int rc = allocation_base(dev_ptr, &base);
  if (rc != EIR_SUCCESS) return rc;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, base);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == EIR_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<char const *>(dev_ptr) - base;
  return EIR_SUCCESS;
}

int eir_ipc_open_handle(void const *handle, int64_t offset, void **dev_ptr, void **base) {
  if (handle == nullptr || dev_ptr == nullptr || base == nullptr || offset < 0)
    return set_error(EIR_INVALID_ARGUMENT, "bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void *b = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *base = b;
  *dev_ptr = static_cast<char *>(b) + offset;
  return EIR_SUCCESS;
}

int eir_ipc_close_handle(void *base) {
  if (base == nullptr) return EIR_SUCCESS;
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return EIR_SUCCESS;
}

int64_t eir_contract_num_ops(eir_plan const *p) { return (p && p->what == 1) ? p->num_ops : 0; }

int eir_permute_plan_create(int32_t nd, int64_t const *sizes, int64_t const *sin,
                            int64_t const *sout, int32_t dtype, eir_plan **plan_out) {
  if (plan_out == nullptr) return set_error(EIR_INVALID_ARGUMENT, "null plan pointer");
  *plan_out = nullptr;
  if (nd < 0 || (nd > 0 && (sizes == nullptr || sin == nullptr || sout == nullptr)))
    return set_error(EIR_INVALID_ARGUMENT, "bad permute dims");
  int64_t es = dtype_bytes(dtype);
  if (es < 0) return set_error(EIR_INVALID_DTYPE, "unsupported permute dtype");
  eir_plan *p = new eir_plan();
  p->what = 2;
  p->family = EIR_FAMILY_PERMUTE;
  p->esize = (int)es;
  int rc = plan_permute(nd, sizes, sin, sout, (int)es, &p->perm, &p->text);
  if (rc != EIR_SUCCESS) {
    delete p;
    return rc;
  }
  *plan_out = p;
  return EIR_SUCCESS;
}

int eir_unary_plan_create(int32_t nd, int64_t const *sizes, int64_t const *sin, int64_t const *sout,
                          int32_t dtype, int32_t ktype, eir_plan **plan_out) {
  if (ktype == EIR_KTYPE_COPY) return eir_permute_plan_create(nd, sizes, sin, sout, dtype, plan_out);
  if (plan_out == nullptr) return set_error(EIR_INVALID_ARGUMENT, "null plan pointer");
  *plan_out = nullptr;
  if (ktype != EIR_KTYPE_ZERO) return set_error(EIR_INVALID_KTYPE, "unary kernel must be COPY or ZERO");
  // ZERO: a row plan over the output's strides alone
  int rc = eir_permute_plan_create(nd, sizes, sout, sout, dtype, plan_out);
  if (rc != EIR_SUCCESS) return rc;
  (*plan_out)->unary_zero = true;
  (*plan_out)->text = "zero: " + (*plan_out)->text;
  return EIR_SUCCESS;
}

int eir_permute(eir_plan *p, void const *in, void *out, void *stream) {
  if (p == nullptr || p->what != 2) return set_error(EIR_INVALID_ARGUMENT, "not a permute plan");
  if (p->perm.total == 0) return EIR_SUCCESS;
  if ((in == nullptr && !p->unary_zero) || out == nullptr)
    return set_error(EIR_NO_DATA_PTR_PROVIDED, "null pointer");
  DeviceState *ds = nullptr;
  int rc = device_state(&ds);
  if (rc != EIR_SUCCESS) return rc;
  return run_permute(p, in, out, ds->num_sms, static_cast<cudaStream_t>(stream));
}

int eir_plan_profile(eir_plan *p, int32_t enable) {
  if (p == nullptr) return set_error(EIR_INVALID_ARGUMENT, "null plan");
  p->profile = enable != 0;
  return EIR_SUCCESS;
}

int eir_plan_profile_read(eir_plan *p, double *ms_total, int64_t *launches) {
  if (p == nullptr) return set_error(EIR_INVALID_ARGUMENT, "null plan");
  double tot = 0.0;
  for (size_t i = 0; i < p->prof_used; ++i) {
    cudaError_t e = cudaEventSynchronize(p->prof_events[i].second);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventSynchronize");
    float ms = 0.f;
    e = cudaEventElapsedTime(&ms, p->prof_events[i].first, p->prof_events[i].second);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventElapsedTime");
    tot += ms;
  }
  if (ms_total) *ms_total = tot;
  if (launches) *launches = (int64_t)p->prof_used;
  p->prof_used = 0;
  return EIR_SUCCESS;
}

int eir_plan_destroy(eir_plan *p) {
  if (p == nullptr) return EIR_SUCCESS;
  for (auto &ev : p->prof_events) {
    cudaEventDestroy(ev.first);
    cudaEventDestroy(ev.second);
  }
  if (p->pre_l) eir_plan_destroy(p->pre_l);
  if (p->pre_r) eir_plan_destroy(p->pre_r);
  if (p->cpx_inner) eir_plan_destroy(p->cpx_inner);
  release_gather(p);
  if (p->ws) {
    int cur = 0;
    cudaGetDevice(&cur);
    if (p->ws_device >= 0 && p->ws_device != cur) cudaSetDevice(p->ws_device);
    cudaFree(p->ws);
    if (p->ws_device >= 0 && p->ws_device != cur) cudaSetDevice(cur);
  }
  delete p;
  return EIR_SUCCESS;
}

int eir_plan_kernel_family(eir_plan const *p) { return p ? p->family : EIR_FAMILY_NONE; }

int64_t eir_plan_workspace_bytes(eir_plan const *p) { return p ? p->ws_bytes : 0; }

char const *eir_plan_describe(eir_plan const *p) { return p ? p->text.c_str() : ""; }

int eir_check_device_errors(void *stream) {
  // no device state is created here (a caller of eir_contract_no_alloc may
  // use this without allocating): the words that exist are read and cleared
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  uint32_t *words[2] = {nullptr, eir::noalloc_error_word(dev)};
  if (dev >= 0 && dev < 64) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    words[0] = g_dev[dev].err;
  }
  uint32_t code = 0;
  for (uint32_t *w : words) {
    if (w == nullptr) continue;
    uint32_t h = 0;
    e = cudaMemcpy(&h, w, sizeof(h), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(error word)");
    if (h != 0) {
      e = cudaMemset(w, 0, sizeof(uint32_t));
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(error word)");
      if (code == 0) code = h;
    }
  }
  if (code != 0) {
    char buf[96];
    std::snprintf(buf, sizeof(buf), "device wait timed out (code 0x%x)", code);
    return set_error(EIR_DEVICE_TIMEOUT, buf);
  }
  return EIR_SUCCESS;
}

}  // extern "C"
