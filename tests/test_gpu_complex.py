"""Complex contractions (EIR_DIM_CPX + CPX_ZERO / CPX_MADD, the reference's
dim_t::CPX and kernel_t::CPX_* ; BinaryContraction.cpp:453-462): the complex
dim (size 2: real, imaginary) sits in left, right and out, either innermost
(interleaved, BATCH_INNER) or outermost (planar). Checked against numpy's
complex128 einsum of the same values; FP32 results within 1e-5 relative
(FP32-exact compute), FP64 within 1e-12."""
from __future__ import annotations

import numpy as np
import pytest

from einsum_ir_b200 import binary, cabi


def _dims(expr, sizes):
    """expr with the complex dim named 'x' -> (ids, eir dims, names)"""
    il, ir, io, names = binary.parse_binary(expr)
    sz = {i: sizes.get(c, 2) for i, c in enumerate(names)}
    dims = binary.contraction_dims(il, ir, io, sz, cpx_id=names.index("x"))
    return il, ir, io, names, sz, dims


def _complex_view(a, ids, names):
    """real array with a size-2 'x' axis -> complex array without it"""
    ax = [names[i] for i in ids].index("x")
    a = np.moveaxis(a, ax, -1)
    return a[..., 0] + 1j * a[..., 1]


def test_complex_plan_structure():
    il, ir, io, names, sz, dims = _dims("xmk,xnk->xnm", dict(m=32, n=24, k=16))
    plan = cabi.ContractPlan(dims, cabi.FP32, cabi.FP32, cabi.FP32, 0, cabi.KTYPE_CPX_ZERO,
                             cabi.KTYPE_CPX_MADD)
    # the reference's count: 2 C M N K * 2 (complex multiply) - C M N, C including the complex 2
    c, m, n, k = 2, 32, 24, 16
    assert plan.num_ops == 2 * c * m * n * k * 2 - c * m * n
    assert plan.describe().startswith("complex:")
    bad = [d if d[0] != cabi.DIM_CPX else (cabi.DIM_CPX, 3) + d[2:] for d in dims]
    with pytest.raises(cabi.EirError) as e:
        cabi.ContractPlan(bad, cabi.FP32, cabi.FP32, cabi.FP32, 0, cabi.KTYPE_CPX_ZERO, cabi.KTYPE_CPX_MADD)
    assert e.value.code == 8  # INVALID_CPX_DIM
    with pytest.raises(cabi.EirError) as e:
        cabi.ContractPlan(dims, cabi.FP32, cabi.FP32, cabi.FP32, 0, cabi.KTYPE_ZERO, cabi.KTYPE_MADD)
    assert e.value.code == 10  # INVALID_KTYPE


CASES = [
    ("mkx,nkx->nmx", dict(m=64, n=48, k=40), "fp32"),          # interleaved (BATCH_INNER)
    ("mkx,nkx->nmx", dict(m=64, n=48, k=40), "fp64"),
    ("xmk,xnk->xnm", dict(m=256, n=256, k=256), "fp32"),        # planar: tensor-core inner problem
    ("xmk,xnk->xnm", dict(m=256, n=192, k=128), "fp64"),
    ("xbmk,xbnk->xbnm", dict(b=3, m=160, n=96, k=64), "fp32"),  # batch (C) dim
    ("bmkx,bknx->bnmx", dict(b=2, m=48, n=40, k=24), "fp32"),   # interleaved, B MN-major
    ("xak,xkb->xab", dict(a=300, b=200, k=72), "fp32"),
]


@pytest.mark.gpu
@pytest.mark.parametrize("accumulate", [False, True])
@pytest.mark.parametrize("expr,sizes,dtype", CASES)
def test_complex_contraction(cuda, expr, sizes, dtype, accumulate):
    import os
    import torch
    os.environ["EIR_TC_MIN_OPS"] = "0"
    os.environ["EIR_TC_MIN_UTIL"] = "0"
    il, ir, io, names, sz, dims = _dims(expr, sizes)
    dt = cabi.FP64 if dtype == "fp64" else cabi.FP32
    tdt = torch.float64 if dtype == "fp64" else torch.float32
    plan = cabi.ContractPlan(dims, dt, dt, dt, 0,
                             cabi.KTYPE_UNDEFINED if accumulate else cabi.KTYPE_CPX_ZERO,
                             cabi.KTYPE_CPX_MADD)
    g = torch.Generator().manual_seed(5)
    shape = lambda ids: [sz[i] for i in ids]
    l = torch.rand(shape(il), generator=g, dtype=torch.float64) * 2 - 1
    r = torch.rand(shape(ir), generator=g, dtype=torch.float64) * 2 - 1
    o0 = torch.rand(shape(io), generator=g, dtype=torch.float64) * 2 - 1
    l, r, o0 = l.to(tdt), r.to(tdt), o0.to(tdt)
    dout = o0.to(cuda)
    plan.contract(l.to(cuda), r.to(cuda), dout)
    torch.cuda.synchronize()
    cabi.check_device_errors()
    got = _complex_view(dout.cpu().double().numpy(), io, names)
    L = _complex_view(l.double().numpy(), il, names)
    R = _complex_view(r.double().numpy(), ir, names)
    sub = lambda ids: "".join(names[i] for i in ids if names[i] != "x")
    ref = np.einsum(f"{sub(il)},{sub(ir)}->{sub(io)}", L, R)
    if accumulate:
        ref = ref + _complex_view(o0.double().numpy(), io, names)
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err <= (1e-12 if dtype == "fp64" else 1e-5), f"{expr} {dtype}: {err:.3e} | {plan.describe()}"
