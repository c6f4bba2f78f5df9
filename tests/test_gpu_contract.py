"""GPU parity of strided binary contractions (C-ABI) against the CPU oracle.

Cases mirror the reference's numeric tests (BinaryContractionTpp.test.torch.cpp:
matmul, bias broadcasts, batched C dims, ZERO+RELU, permuted operands) and the
BASELINE configs at reduced sizes. Tolerances are relative Frobenius errors
against the oracle evaluated on the same inputs: BF16 inputs with FP32
accumulation 1e-5 (north_star allows 1e-2), FP32-accurate (3xTF32 / SIMT FP32)
1e-5 (north_star: 1e-4), TF32 1e-5 (the kernels round every FP32 operand to
the nearest TF32 value, ties to even, as the oracle's TF32 model does, on
TF32-representable and on general FP32 inputs), FP64 1e-12.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from einsum_ir_b200 import binary, cabi
from tests import _oracle

pytestmark = pytest.mark.gpu

TOL = {"bf16": 1e-5, "fp32": 1e-5, "tf32": 1e-5, "tf32_general": 1e-5, "fp64": 1e-12}


def _make_inputs(torch, shape_l, shape_r, dtype, seed, tf32_exact):
    g = torch.Generator().manual_seed(seed)
    tdt = {"bf16": torch.bfloat16, "fp64": torch.float64}.get(dtype, torch.float32)
    l = (torch.rand(shape_l, generator=g, dtype=torch.float64) * 2 - 1).to(tdt)
    r = (torch.rand(shape_r, generator=g, dtype=torch.float64) * 2 - 1).to(tdt)
    if tf32_exact:
        l = torch.from_numpy(_oracle.round_tf32(l.numpy()))
        r = torch.from_numpy(_oracle.round_tf32(r.numpy()))
    return l.contiguous(), r.contiguous()


def _np_in(t):
    import torch
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).ravel()
    return t.numpy().ravel()


def run_case(cuda, expr, sizes, dtype="fp32", comp=None, first=cabi.KTYPE_ZERO,
             last=cabi.KTYPE_UNDEFINED, aux_outer=None, flags=0, seed=0, expect_family=None,
             tf32_general=False, tc_min_ops="0", pair=None, bn=None, ksub=None, tol=None, direct=None):
    """pair / bn / ksub force the tensor-core tile shape (CTA pair or one CTA,
    BN, K blocks per stage); None leaves the planner's choice. direct: True
    expects the one-output-per-thread CUDA-core kernel, False keeps the tiled
    one. tol overrides the dtype's tolerance."""
    import torch
    os.environ["EIR_TC_MIN_OPS"] = tc_min_ops
    os.environ["EIR_TC_MIN_UTIL"] = "0"
    direct_env = None if direct is None else ("1" if direct else "0")
    for var, val in (("EIR_TC_PAIR", pair), ("EIR_TC_BN", bn), ("EIR_TC_KSUB", ksub),
                     ("EIR_SIMT_DIRECT", direct_env)):
        if val is None:
            os.environ.pop(var, None)
        else:
            os.environ[var] = str(val)
    il, ir, io, names = binary.parse_binary(expr)
    sz = {i: sizes[c] for i, c in enumerate(names)}
    aux_sizes = None
    if aux_outer is not None:
        aux_sizes = {i: (1 if names[i] in aux_outer else sz[i]) for i in sz}
    dims = binary.contraction_dims(il, ir, io, sz, sizes_outer_aux=aux_sizes)
    dt = {"bf16": cabi.BF16, "fp64": cabi.FP64}.get(dtype, cabi.FP32)
    dto = cabi.FP64 if dtype == "fp64" else cabi.FP32
    if comp is None:
        comp = {"tf32": cabi.COMPUTE_TF32}.get(dtype, cabi.COMPUTE_DEFAULT)
    plan = cabi.ContractPlan(dims, dt, dt, dto, comp, first, cabi.KTYPE_MADD, last, flags)
    if expect_family is not None:
        assert plan.family == expect_family, plan.describe()
    if direct is not None:
        assert ("one output per thread" in plan.describe()) == direct, plan.describe()

    shape = lambda ids: [sz[i] for i in ids]
    l, r = _make_inputs(torch, shape(il), shape(ir), dtype, seed,
                        tf32_exact=(dtype == "tf32" and not tf32_general))
    odt = torch.float64 if dtype == "fp64" else torch.float32
    g = torch.Generator().manual_seed(seed + 7)
    out0 = (torch.rand(shape(io), generator=g, dtype=torch.float64) * 2 - 1).to(odt)
    aux = None
    if aux_sizes is not None:
        aux = (torch.rand([aux_sizes[i] for i in io], generator=g, dtype=torch.float64) * 2 - 1).to(odt)

    dl, dr, dout = l.to(cuda), r.to(cuda), out0.to(cuda)
    daux = aux.to(cuda) if aux is not None else None
    plan.contract(dl, dr, dout, daux)
    torch.cuda.synchronize()
    cabi.check_device_errors()
    got = dout.cpu().numpy().ravel()

    ref = out0.numpy().ravel().copy()
    _oracle.contract(dims, _np_in(l), _np_in(r), ref, None if aux is None else aux.numpy().ravel(),
                     dt, dt, dto, comp if dtype != "tf32" else cabi.COMPUTE_TF32, first, last)
    key = "tf32_general" if (dtype == "tf32" and tf32_general) else dtype
    err = _oracle.rel_err(got, ref)
    assert np.all(np.isfinite(got))
    bound = TOL[key] if tol is None else tol
    assert err <= bound, f"{expr} {dtype}: rel err {err:.3e} ({plan.describe()})"
    return plan, err


TC = cabi.FAMILY_TC
SIMT = cabi.FAMILY_SIMT

TC_CASES = [
    # BASELINE config 2 at reduced a/k: K-order mismatch -> right operand pre-permuted
    ("akmj,njk->anm", dict(a=2, k=4, m=128, j=64, n=256), "bf16"),
    ("akmj,njk->anm", dict(a=3, k=5, m=200, j=40, n=130), "bf16"),
    # plain GEMMs, every operand major-ness combination
    ("mk,nk->nm", dict(m=256, n=384, k=192), "bf16"),      # A K-major, B K-major
    ("km,nk->nm", dict(m=256, n=384, k=192), "bf16"),      # A MN-major, B K-major
    ("mk,kn->nm", dict(m=256, n=384, k=192), "bf16"),      # A K-major, B MN-major
    ("km,kn->nm", dict(m=256, n=384, k=192), "bf16"),      # both MN-major
    ("mk,nk->nm", dict(m=130, n=70, k=40), "bf16"),        # ragged tails
    ("km,kn->nm", dict(m=132, n=72, k=33), "fp32"),
    ("mk,nk->nm", dict(m=256, n=256, k=160), "fp32"),
    ("km,nk->nm", dict(m=256, n=256, k=160), "tf32"),
    ("km,kn->nm", dict(m=192, n=320, k=96), "tf32"),
    # BASELINE config 5 at reduced sizes (swap already applied: left = zcdef)
    ("zcdef,zabcd->zabef", dict(z=3, a=8, b=8, c=8, d=8, e=8, f=8), "tf32"),
    ("zcdef,zabcd->zabef", dict(z=3, a=8, b=8, c=8, d=8, e=8, f=8), "fp32"),
    ("zcdef,zabcd->zabef", dict(z=2, a=8, b=6, c=4, d=16, e=8, f=16), "bf16"),
    # non-fusable M dims and C dims inside, tile loops + outer K loops
    ("axmk,nkx->anm", dict(a=3, x=2, m=96, k=64, n=80), "bf16"),
    ("cmk,cnk->cnm", dict(c=3, m=128, n=192, k=128), "fp32"),
    ("abmkq,cnqk->acbnm", dict(a=2, b=3, c=2, m=64, n=48, k=16, q=8), "bf16"),
]


@pytest.mark.parametrize("expr,sizes,dtype", TC_CASES)
def test_tc_parity(cuda, expr, sizes, dtype):
    run_case(cuda, expr, sizes, dtype, expect_family=TC)


def _m_size(expr, sizes):
    """size of the primitive M dim the planner picks: the output's fastest M dim"""
    il, ir, io, names = binary.parse_binary(expr)
    return sizes[names[[i for i in io if i in il][-1]]]


@pytest.mark.parametrize("pair", [0, 1])
@pytest.mark.parametrize("expr,sizes,dtype", TC_CASES)
def test_tc_parity_tile_shapes(cuda, expr, sizes, dtype, pair):
    """Every tensor-core case on the one-CTA kernel and on CTA pairs (cta_group::2)."""
    plan, _ = run_case(cuda, expr, sizes, dtype, expect_family=TC, pair=pair)
    assert ("pair" in plan.describe()) == (pair == 1 and _m_size(expr, sizes) > 128), plan.describe()


PAIR_CASES = [
    # M = 300: the second pair tile's odd CTA reads only rows past the end (TMA zero fill)
    ("mk,nk->nm", dict(m=300, n=200, k=96), "bf16", 256, 2),
    ("mk,nk->nm", dict(m=300, n=200, k=96), "bf16", 128, 1),
    ("km,kn->nm", dict(m=384, n=136, k=72), "bf16", 128, 2),
    ("km,kn->nm", dict(m=260, n=520, k=40), "tf32", 256, 1),
    ("mk,kn->nm", dict(m=512, n=256, k=256), "tf32", 128, 1),
    # FP32-exact (3xTF32) on pairs: hi / lo split by each CTA's converter warps
    ("mk,nk->nm", dict(m=300, n=200, k=96), "fp32", 256, 1),
    ("km,kn->nm", dict(m=384, n=136, k=72), "fp32", 128, 1),
    ("zcdef,zabcd->zabef", dict(z=3, a=16, b=8, c=8, d=8, e=16, f=16), "fp32", 256, 1),
    # several tiles per pair (persistent loop, accumulator double buffering)
    ("cmk,cnk->cnm", dict(c=40, m=512, n=512, k=128), "bf16", 256, 2),
    ("akmj,njk->anm", dict(a=4, k=8, m=512, j=64, n=512), "bf16", 256, 2),
    ("cmk,cnk->cnm", dict(c=12, m=512, n=512, k=64), "fp32", 256, 1),
]


@pytest.mark.parametrize("expr,sizes,dtype,bn,ksub", PAIR_CASES)
def test_tc_pair_shapes(cuda, expr, sizes, dtype, bn, ksub):
    plan, _ = run_case(cuda, expr, sizes, dtype, expect_family=TC, pair=1, bn=bn, ksub=ksub)
    d = plan.describe()
    assert "pair" in d and f"BN={bn} KSUB={ksub}" in d, d


# Long K: the accumulation runs in chunks (1024 K for FP32-exact, 8192 K for
# TF32 and BF16) that the epilogue adds in FP32; a single TMEM accumulation
# over these K would drift past 1e-5 (about 2e-8 per accumulating MMA).
LONG_K_CASES = [
    ("mk,nk->nm", dict(m=128, n=256, k=16384), "fp32"),
    ("km,kn->nm", dict(m=200, n=136, k=3000), "fp32"),           # ragged, partial last chunk
    ("mkx,nkx->nm", dict(m=256, n=128, k=96, x=64), "fp32"),     # K = primitive x outer loop
    ("mk,nk->nm", dict(m=128, n=256, k=12288), "tf32"),
    ("mk,nk->nm", dict(m=128, n=256, k=32768), "bf16"),
]
LONG_K_TOUCH = [(cabi.KTYPE_ZERO, cabi.KTYPE_UNDEFINED, None),
                (cabi.KTYPE_UNDEFINED, cabi.KTYPE_RELU, None),      # accumulate into out
                (cabi.KTYPE_COPY, cabi.KTYPE_RELU, "m"),            # bias along n
                (cabi.KTYPE_ADD, cabi.KTYPE_ADD, "n")]


@pytest.mark.parametrize("pair", [0, 1])
@pytest.mark.parametrize("first,last,aux", LONG_K_TOUCH)
@pytest.mark.parametrize("expr,sizes,dtype", LONG_K_CASES)
def test_tc_long_k_chunks(cuda, expr, sizes, dtype, first, last, aux, pair):
    # FP32-exact keeps its 1e-5; TF32 and BF16 chunks are long (8192 K, up to
    # 1024 accumulating MMAs) and are held to north_star's FP32/TF32 1e-4
    run_case(cuda, expr, sizes, dtype, first=first, last=last, aux_outer=aux, expect_family=TC,
             pair=pair, tol=1e-5 if dtype == "fp32" else 1e-4)


# Split-K: few output tiles and a long K walk run as K slices (one-CTA
# kernel, partial tiles in a workspace) summed by a reduction kernel, which
# applies the touch kernels.
SPLITK_CASES = [
    ("mk,nk->nm", dict(m=128, n=128, k=16384), "fp32"),
    ("km,kn->nm", dict(m=200, n=136, k=8192), "bf16"),
    ("cmk,cnk->cnm", dict(c=2, m=128, n=96, k=6000), "tf32"),     # tile loop, ragged K
    ("mkx,nkx->nm", dict(m=96, n=128, k=64, x=96), "fp32"),       # K = primitive x outer loop
]


@pytest.mark.parametrize("first,last,aux", LONG_K_TOUCH)
@pytest.mark.parametrize("expr,sizes,dtype", SPLITK_CASES)
def test_tc_split_k(cuda, expr, sizes, dtype, first, last, aux):
    plan, _ = run_case(cuda, expr, sizes, dtype, first=first, last=last, aux_outer=aux,
                       expect_family=TC, tol=1e-4 if dtype == "tf32" else 1e-5)
    d = plan.describe()
    assert "splitk=" in d and "splitk=1 " not in d and "pair" not in d, d


@pytest.mark.parametrize("expr,pair", [("km,nk->nm", 0), ("km,nk->nm", 1), ("mk,kn->nm", 1),
                                       ("zcdef,zabcd->zabef", None)])
def test_tc_tf32_general_inputs(cuda, expr, pair):
    # general FP32 inputs: the kernels round every operand to the nearest TF32
    # value (ties to even) in shared memory, the oracle's TF32 model
    sizes = dict(m=256, n=256, k=256) if "m" in expr else dict(z=3, a=8, b=8, c=8, d=8, e=8, f=8)
    run_case(cuda, expr, sizes, "tf32", tf32_general=True, expect_family=TC, pair=pair)


def test_simt_tf32_general_inputs(cuda):
    # the CUDA-core kernel rounds its TF32 operands as they are loaded
    run_case(cuda, "zab,zbc->zac", dict(z=5, a=7, b=9, c=6), "tf32", tf32_general=True,
             expect_family=SIMT, tc_min_ops=str(1 << 40))


@pytest.mark.parametrize("expr,sizes,dtype", [
    ("mk,nk->mn", dict(m=256, n=384, k=192), "bf16"),
    ("mk,kn->mn", dict(m=256, n=384, k=96), "fp32"),
    ("km,kn->mn", dict(m=200, n=130, k=64), "tf32"),
    ("zabcd,zcdef->zabef", dict(z=3, a=8, b=8, c=8, d=8, e=8, f=8), "fp32"),
    ("zabcd,zcdef->zabef", dict(z=3, a=8, b=8, c=8, d=8, e=8, f=8), "fp64"),
])
def test_tc_output_contiguous_along_right_operand(cuda, expr, sizes, dtype):
    # the output's unit-stride dim belongs to the right operand: the plan swaps
    # the operand roles (the reference's swap_inputs rule) and the result stays
    plan, _ = run_case(cuda, expr, sizes, dtype)
    assert "operands swapped" in plan.describe(), plan.describe()


@pytest.mark.parametrize("dtype", ["fp32", "bf16", "fp64"])
def test_swapped_mlp_layer_bias_relu(cuda, dtype):
    # bi,io->bo: bias broadcast over b, output contiguous along o (right operand)
    plan, _ = run_case(cuda, "bi,io->bo", dict(b=256, i=192, o=320), dtype, first=cabi.KTYPE_COPY,
                       last=cabi.KTYPE_RELU, aux_outer="b")
    assert "operands swapped" in plan.describe(), plan.describe()


@pytest.mark.parametrize("dtype", ["fp32", "bf16", "tf32"])
@pytest.mark.parametrize("pair", [0, 1])
def test_tc_mlp_layer_bias_relu(cuda, dtype, pair):
    # bench_mlp hidden layer: COPY bias (broadcast over b) first touch, RELU last touch
    run_case(cuda, "io,bi->bo", dict(b=256, i=192, o=320), dtype, first=cabi.KTYPE_COPY,
             last=cabi.KTYPE_RELU, aux_outer="b", expect_family=TC, pair=pair)


@pytest.mark.parametrize("first,last", [(cabi.KTYPE_UNDEFINED, cabi.KTYPE_UNDEFINED),
                                        (cabi.KTYPE_ADD, cabi.KTYPE_UNDEFINED),
                                        (cabi.KTYPE_ZERO, cabi.KTYPE_ADD),
                                        (cabi.KTYPE_COPY, cabi.KTYPE_ADD)])
@pytest.mark.parametrize("pair", [0, 1])
def test_tc_touch_kernels(cuda, first, last, pair):
    run_case(cuda, "mk,nk->nm", dict(m=160, n=96, k=64), "bf16", first=first, last=last,
             aux_outer="n", expect_family=TC, pair=pair)


DMMA = cabi.FAMILY_DMMA

DMMA_CASES = [
    ("mk,nk->nm", dict(m=256, n=384, k=64), "fp64"),        # A K-major, B K-major
    ("km,nk->nm", dict(m=256, n=384, k=48), "fp64"),        # A MN-major, B K-major
    ("mk,kn->nm", dict(m=256, n=384, k=48), "fp64"),        # A K-major, B MN-major
    ("km,kn->nm", dict(m=256, n=384, k=80), "fp64"),        # both MN-major
    ("mk,nk->nm", dict(m=130, n=70, k=34), "fp64"),         # ragged tails
    ("zcdef,zabcd->zabef", dict(z=3, a=8, b=8, c=8, d=8, e=8, f=8), "fp64"),
    ("axmk,nkx->anm", dict(a=3, x=2, m=96, k=64, n=80), "fp64"),
]


@pytest.mark.parametrize("expr,sizes,dtype", DMMA_CASES)
def test_dmma_parity(cuda, expr, sizes, dtype):
    run_case(cuda, expr, sizes, dtype, expect_family=DMMA)


def test_dmma_bias_relu(cuda):
    run_case(cuda, "io,bi->bo", dict(b=256, i=96, o=192), "fp64", first=cabi.KTYPE_COPY,
             last=cabi.KTYPE_RELU, aux_outer="b", expect_family=DMMA)


SIMT_CASES = [
    ("bf,dcba->acdf", dict(a=4, b=3, c=5, d=8, f=2), "fp32"),
    ("dh,acdf->acfh", dict(a=4, c=5, d=8, f=2, h=9), "fp32"),
    ("iae,cg->acegi", dict(a=4, c=5, e=7, g=3, i=6), "fp32"),     # K = empty (outer product)
    ("acfh,acegi->hgfei", dict(a=4, c=5, e=7, f=2, g=3, h=9, i=6), "fp32"),
    ("zcdef,zabcd->zabef", dict(z=3, a=5, b=4, c=6, d=3, e=7, f=2), "fp64"),
    ("mk,nk->nm", dict(m=67, n=45, k=29), "fp64"),
    ("km,kn->nm", dict(m=67, n=45, k=29), "bf16"),
    ("cmk,cnk->cnm", dict(c=3, m=17, n=19, k=23), "fp32"),
    ("abmkq,cnqk->abcnm", dict(a=2, b=2, c=2, m=64, n=64, k=32, q=3), "bf16"),
]


# the cases the planner gives the one-output-per-thread kernel (fewer than
# 2^22 outputs, K <= 64 or outputs x K <= 2^16); the last SIMT case (K = 96,
# 32768 outputs) stays on the tiled kernel
SIMT_DIRECT_CASES = SIMT_CASES[:-1]


@pytest.mark.parametrize("expr,sizes,dtype", SIMT_CASES)
def test_simt_parity(cuda, expr, sizes, dtype):
    # the tiled 64 x 64 kernel (the direct kernel switched off)
    run_case(cuda, expr, sizes, dtype, flags=cabi.FLAG_FORCE_SIMT, expect_family=SIMT, direct=False)


@pytest.mark.parametrize("expr,sizes,dtype", SIMT_DIRECT_CASES)
def test_simt_direct_parity(cuda, expr, sizes, dtype):
    run_case(cuda, expr, sizes, dtype, flags=cabi.FLAG_FORCE_SIMT, expect_family=SIMT, direct=True)


def test_simt_default_choice(cuda):
    # the planner's own choice (no override): tiled for the K = 96 case
    run_case(cuda, *SIMT_CASES[-1], flags=cabi.FLAG_FORCE_SIMT, expect_family=SIMT)


@pytest.mark.parametrize("expr,sizes,dtype", [
    ("mk,nk->nm", dict(m=2, n=2, k=16384), "fp32"),      # 64 accumulation chunks of 256
    ("mk,nk->nm", dict(m=2, n=2, k=16384), "fp64"),
    ("abkq,qk->ab", dict(a=3, b=4, k=1000, q=5), "fp32"),  # two K dims, the outer one walked
    ("zab,zbc->zac", dict(z=5, a=7, b=9, c=6), "bf16"),
])
def test_simt_direct_long_k(cuda, expr, sizes, dtype):
    run_case(cuda, expr, sizes, dtype, flags=cabi.FLAG_FORCE_SIMT, expect_family=SIMT, direct=True)


@pytest.mark.parametrize("first,last", [(cabi.KTYPE_UNDEFINED, cabi.KTYPE_UNDEFINED),
                                        (cabi.KTYPE_ADD, cabi.KTYPE_UNDEFINED),
                                        (cabi.KTYPE_ZERO, cabi.KTYPE_ADD),
                                        (cabi.KTYPE_COPY, cabi.KTYPE_RELU)])
def test_simt_direct_touches(cuda, first, last):
    run_case(cuda, "mk,nk->nm", dict(m=33, n=17, k=9), "fp32", first=first, last=last, aux_outer="n",
             flags=cabi.FLAG_FORCE_SIMT, expect_family=SIMT, direct=True)


def test_simt_direct_tf32_general_inputs(cuda):
    run_case(cuda, "zab,zbc->zac", dict(z=5, a=7, b=9, c=6), "tf32", tf32_general=True,
             flags=cabi.FLAG_FORCE_SIMT, expect_family=SIMT, direct=True)


def test_simt_long_k(cuda):
    """K = 65536 on the CUDA cores: chunked FP32 accumulation keeps the error
    near 2e-6 (a single FP32 running sum drifts to ~1.5e-5)"""
    run_case(cuda, "mk,nk->nm", dict(m=64, n=96, k=65536), "fp32", flags=cabi.FLAG_FORCE_SIMT,
             expect_family=SIMT)


@pytest.mark.parametrize("dtype", ["fp32", "fp64"])
def test_simt_bias_relu_fp(cuda, dtype):
    run_case(cuda, "io,bi->bo", dict(b=33, i=20, o=41), dtype, first=cabi.KTYPE_COPY,
             last=cabi.KTYPE_RELU, aux_outer="b", flags=cabi.FLAG_FORCE_SIMT,
             expect_family=SIMT)


def test_size_zero_and_one_dims(cuda):
    import torch
    # a size-0 M dim: nothing to do, output untouched
    dims = [(cabi.DIM_M, 0, 1, 0, 1, 0), (cabi.DIM_N, 8, 0, 1, 0, 0), (cabi.DIM_K, 4, 0, 8, 0, 0)]
    plan = cabi.ContractPlan(dims, cabi.FP32, cabi.FP32, cabi.FP32)
    out = torch.ones(4, device=cuda)
    plan.contract(torch.zeros(1, device=cuda), torch.zeros(32, device=cuda), out)
    torch.cuda.synchronize()
    assert torch.all(out == 1)
    # size-1 dims everywhere
    run_case(cuda, "amk,bnk->abnm", dict(a=1, b=1, m=33, n=17, k=9), "fp32")
