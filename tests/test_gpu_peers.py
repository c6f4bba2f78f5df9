"""Peer outputs (eir_contract_peers): the epilogue of every kernel family
stores the final output into `out` and into each peer output at the same
offsets. On one GPU the peers are other buffers of the same device (the
kernels store through plain pointers, local or mapped from another GPU
alike); every copy must equal `out` bit for bit and `out` the oracle."""
from __future__ import annotations

import os

import numpy as np
import pytest

from einsum_ir_b200 import binary, cabi
from tests import _oracle

pytestmark = pytest.mark.gpu

CASES = [
    # (expr, sizes, dtype, family, flags)
    ("mk,nk->nm", dict(m=256, n=384, k=192), "bf16", cabi.FAMILY_TC, 0),
    ("km,kn->nm", dict(m=300, n=200, k=96), "fp32", cabi.FAMILY_TC, 0),
    ("mk,nk->nm", dict(m=128, n=256, k=4096), "fp32", cabi.FAMILY_TC, 0),      # 4 accumulation chunks
    ("zcdef,zabcd->zabef", dict(z=2, a=8, b=8, c=8, d=8, e=16, f=16), "fp64", cabi.FAMILY_DMMA, 0),
    ("mk,nk->nm", dict(m=70, n=50, k=40), "fp32", cabi.FAMILY_SIMT, cabi.FLAG_FORCE_SIMT),
    ("akmj,njk->anm", dict(a=2, k=4, m=128, j=64, n=256), "bf16", cabi.FAMILY_TC, 0),  # pre-permute
    ("mk,nk->nm", dict(m=128, n=128, k=16384), "fp32", cabi.FAMILY_TC, 0),  # split-K: the reduction stores
]


@pytest.mark.parametrize("peers", [1, 3, 7])
@pytest.mark.parametrize("expr,sizes,dtype,family,flags", CASES)
def test_peer_outputs(cuda, expr, sizes, dtype, family, flags, peers):
    import torch
    os.environ["EIR_TC_MIN_OPS"] = "0"
    os.environ["EIR_TC_MIN_UTIL"] = "0"
    il, ir, io, names = binary.parse_binary(expr)
    sz = {i: sizes[c] for i, c in enumerate(names)}
    dims = binary.contraction_dims(il, ir, io, sz)
    dt = {"bf16": cabi.BF16, "fp64": cabi.FP64}.get(dtype, cabi.FP32)
    dto = cabi.FP64 if dtype == "fp64" else cabi.FP32
    plan = cabi.ContractPlan(dims, dt, dt, dto, 0, cabi.KTYPE_ZERO, cabi.KTYPE_MADD, cabi.KTYPE_RELU, flags)
    assert plan.family == family, plan.describe()
    g = torch.Generator().manual_seed(3)
    tdt = {"bf16": torch.bfloat16, "fp64": torch.float64}.get(dtype, torch.float32)
    odt = torch.float64 if dtype == "fp64" else torch.float32
    shape = lambda ids: [sz[i] for i in ids]
    l = (torch.rand(shape(il), generator=g, dtype=torch.float64) * 2 - 1).to(tdt)
    r = (torch.rand(shape(ir), generator=g, dtype=torch.float64) * 2 - 1).to(tdt)
    out = torch.full(shape(io), float("nan"), dtype=odt, device=cuda)
    copies = [torch.full(shape(io), float("nan"), dtype=odt, device=cuda) for _ in range(peers)]
    plan.contract_peers(l.to(cuda), r.to(cuda), out, copies)
    torch.cuda.synchronize()
    cabi.check_device_errors()
    for c in copies:
        assert torch.equal(c, out)
    ref = np.zeros(out.numel(), dtype=np.float64 if dtype == "fp64" else np.float32)
    npin = (lambda t: t.view(torch.int16).numpy().view(np.uint16).ravel()) if dtype == "bf16" else \
        (lambda t: t.numpy().ravel())
    _oracle.contract(dims, npin(l), npin(r), ref, None, dt, dt, dto, 0, cabi.KTYPE_ZERO, cabi.KTYPE_RELU)
    err = _oracle.rel_err(out.cpu().numpy().ravel(), ref)
    assert err <= (1e-12 if dtype == "fp64" else 1e-5), f"{err:.3e} {plan.describe()}"


def test_peer_argument_errors(cuda):
    import torch
    dims = binary.contraction_dims(*binary.parse_binary("mk,nk->nm")[:3], {0: 8, 1: 8, 2: 8})
    plan = cabi.ContractPlan(dims, cabi.FP32, cabi.FP32, cabi.FP32, 0)
    x = torch.zeros(64, device=cuda)
    with pytest.raises(cabi.EirError):
        plan.contract_peers(x, x, x, [x] * 8)
    with pytest.raises(cabi.EirError):
        plan.contract_peers(x, x, x, [None])


def test_ipc_handle_of_an_allocation(cuda):
    import torch
    buf = torch.zeros(1 << 20, device=cuda)
    h, off = cabi.ipc_get_handle(buf[1000:])
    assert len(h) == cabi.IPC_HANDLE_BYTES and off >= 4000 and off % 4 == 0
