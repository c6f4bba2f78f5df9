// Host-callable launchers of the device kernels (internal to the library).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include "eir_params.h"

namespace eir {

cudaError_t launch_simt_contract(int dt_l, int dt_r, int dt_o, SimtParams const &p, void const *l,
                                 void const *r, void const *aux, void *out, cudaStream_t st);

// the direct (one output per thread) CUDA-core contraction of tiny problems
cudaError_t launch_simt_direct(int dt_l, int dt_r, int dt_o, DirectParams const &p, void const *l,
                               void const *r, void const *aux, void *out, cudaStream_t st);

// split-K reduction of a split tcgen05 plan (TcParams::split_k): p is the
// plan's real parameter block (output strides and touches), ws the workspace
cudaError_t launch_splitk_reduce(TcParams const &p, float const *ws, float const *aux, float *out,
                                 int num_sms, cudaStream_t st);

// zero: the unary ZERO primitive (out = 0 over p's output strides, `in` unused;
// p must be a row-copy plan, which planning with sin = sout gives)
cudaError_t launch_permute(int esize, PermuteParams const &p, void const *in, void *out,
                           int num_sms, cudaStream_t st, bool zero = false);

// right operand of a complex contraction expanded into the real blocks
// [[Br, Bi], [-Bi, Br]] (esize 4 or 8; p: B's non-complex dims, packed sout)
cudaError_t launch_cpx_expand(int esize, PermuteParams const &p, int64_t cpx_stride, void const *in,
                              void *out, int num_sms, cudaStream_t st);

// kind: 0 = BF16 (kind::f16), 1 = TF32, 2 = 3xTF32 (FP32-accurate)
// ksub: K blocks (128-byte swizzle rows) per ring stage, 1 or 2
cudaError_t launch_tc_contract(int kind, int bn, int ksub, bool a_mn, bool b_mn,
                               CUtensorMap const &ma, CUtensorMap const &mb, TcParams const &p,
                               float const *aux, float *out, int num_sms, cudaStream_t st);

// CTA pairs (cta_group::2): 256 x BN tiles, each CTA stages half of A's and
// half of B's rows; kind 0 or 1 (bn 128 or 256, ksub 1 or 2) or 2 (3xTF32,
// bn 128 or 256, ksub 1)
cudaError_t launch_tc_pair_contract(int kind, int bn, int ksub, bool a_mn, bool b_mn,
                                    CUtensorMap const &ma, CUtensorMap const &mb, TcParams const &p,
                                    float const *aux, float *out, cudaStream_t st);

// FP64 on the FP64 tensor cores (mma.sync m8n8k4), 128 x 128 tiles, K blocks of 16
cudaError_t launch_dmma_contract(bool a_mn, bool b_mn, CUtensorMap const &ma, CUtensorMap const &mb,
                                 TcParams const &p, double const *aux, double *out, int num_sms,
                                 cudaStream_t st);

// gathered contraction: sets ctr[0 .. n) to at least `value` after the
// previous kernel of the stream has completed
cudaError_t launch_slab_release(uint32_t *ctr, int32_t n, uint32_t value, cudaStream_t st);

// K elements per block (one 128-byte swizzle row): 64 BF16, 32 FP32/TF32, 16 FP64
int tc_block_k(int kind);

}  // namespace eir
