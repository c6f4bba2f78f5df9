"""eir_contract_gather on one GPU, through the C-ABI.

The entry point contracts a rank's block of a batch-sharded contraction and
copies the finished output, slab by slab of its outermost dim, into other
buffers (the other ranks' outputs on a node). Here the "peers" are buffers on
the same GPU, which exercises everything but NVLink: the per-slab counters the
FP64 DMMA kernel publishes, the copy streams that wait on them, the release
after the kernel (which also serves the kernel families that do not count),
two calls in a row, and two emulated ranks that fill each other's full
outputs. Results are checked against the C oracle (FP64 1e-12, FP32 1e-5
relative) and the peer copies bit for bit."""
from __future__ import annotations

import numpy as np
import pytest

from einsum_ir_b200 import binary, cabi
from tests import _oracle

pytestmark = pytest.mark.gpu


def _setup(expr, sizes, dtype, comp=cabi.COMPUTE_DEFAULT):
    il, ir, io, names = binary.parse_binary(expr)
    sz = {i: sizes[c] for i, c in enumerate(names)}
    dims = binary.contraction_dims(il, ir, io, sz)
    dto = cabi.FP64 if dtype == cabi.FP64 else cabi.FP32
    plan = cabi.ContractPlan(dims, dtype, dtype, dto, comp)
    return plan, dims, [sz[i] for i in il], [sz[i] for i in ir], [sz[i] for i in io]


def _oracle_out(dims, l, r, dtype, comp=cabi.COMPUTE_DEFAULT):
    dto = cabi.FP64 if dtype == cabi.FP64 else cabi.FP32
    ref = np.zeros(int(np.prod([d[1] for d in dims if d[0] != cabi.DIM_K])),
                   dtype=np.float64 if dtype == cabi.FP64 else np.float32)
    _oracle.contract(dims, l.cpu().numpy().ravel(), r.cpu().numpy().ravel(), ref, None, dtype, dtype,
                     dto, comp)
    return ref


@pytest.mark.parametrize("expr,sizes,dtype,family,counted", [
    # FP64 on the DMMA kernel: z is the slowest tile loop, the kernel counts slabs
    ("zabcd,zcdef->zabef", dict(z=4, a=16, b=16, c=16, d=16, e=16, f=16), cabi.FP64, cabi.FAMILY_DMMA, True),
    # ragged tiles (M = N = 400: a partial 128-row tile per slab) and 3 slabs
    ("zabcd,zcdef->zabef", dict(z=3, a=20, b=20, c=16, d=16, e=20, f=20), cabi.FP64, cabi.FAMILY_DMMA, True),
    # the batch dim is not a tile loop of the kernel: one slab, released after the kernel
    ("mk,nk->nm", dict(m=256, n=384, k=512), cabi.FP64, cabi.FAMILY_DMMA, False),
    # tcgen05 (FP32-exact) and the CUDA-core kernel do not count: released after the kernel
    ("zabcd,zcdef->zabef", dict(z=4, a=16, b=16, c=16, d=16, e=16, f=16), cabi.FP32, cabi.FAMILY_TC, False),
    ("zab,zbc->zac", dict(z=5, a=7, b=9, c=6), cabi.FP32, cabi.FAMILY_SIMT, False),
])
def test_gather_matches_oracle_and_peers_match_out(cuda, expr, sizes, dtype, family, counted):
    import torch
    plan, dims, sl, sr, so = _setup(expr, sizes, dtype)
    assert plan.family == family, plan.describe()
    assert ("counted by the kernel" in plan.describe()) == counted, plan.describe()
    tdt = torch.float64 if dtype == cabi.FP64 else torch.float32
    g = torch.Generator().manual_seed(21)
    peers = [torch.full(so, float("nan"), dtype=tdt, device=cuda) for _ in range(3)]
    out = torch.full(so, float("nan"), dtype=tdt, device=cuda)
    for call in range(2):  # two calls in a row: the counters and copy streams are reused
        l = ((torch.rand(sl, generator=g, dtype=torch.float64) * 2 - 1).to(tdt)).to(cuda)
        r = ((torch.rand(sr, generator=g, dtype=torch.float64) * 2 - 1).to(tdt)).to(cuda)
        plan.contract_gather(l, r, out, peers)
        torch.cuda.synchronize()
        cabi.check_device_errors()
        ref = _oracle_out(dims, l, r, dtype)
        err = _oracle.rel_err(out.cpu().numpy(), ref)
        assert err <= (1e-12 if dtype == cabi.FP64 else 1e-5), f"call {call}: {err:.3e} {plan.describe()}"
        for p in peers:
            assert torch.equal(p, out), f"call {call}: a peer copy differs"


def test_gather_two_emulated_ranks(cuda):
    """two 'ranks' on one GPU, each contracting its z block of config 5
    (reduced) into its full output and the other's: both full outputs end
    equal to the whole contraction"""
    import torch
    S = dict(z=6, a=16, b=16, c=16, d=16, e=16, f=16)
    world, zb = 2, 3
    plan, dims, sl, sr, so = _setup("zabcd,zcdef->zabef", dict(S, z=zb), cabi.FP64)
    _, dims_full, sl_f, sr_f, so_f = _setup("zabcd,zcdef->zabef", S, cabi.FP64)
    g = torch.Generator().manual_seed(5)
    L = (torch.rand(sl_f, generator=g, dtype=torch.float64) * 2 - 1).to(cuda)
    R = (torch.rand(sr_f, generator=g, dtype=torch.float64) * 2 - 1).to(cuda)
    outs = [torch.full(so_f, float("nan"), dtype=torch.float64, device=cuda) for _ in range(world)]
    slab_bytes = outs[0][0].numel() * 8
    for rank in range(world):
        z0 = rank * zb
        peer = outs[1 - rank].data_ptr() + z0 * slab_bytes
        plan.contract_gather(L[z0:z0 + zb], R[z0:z0 + zb], outs[rank][z0:z0 + zb], [peer])
    torch.cuda.synchronize()
    cabi.check_device_errors()
    ref = _oracle_out(dims_full, L, R, cabi.FP64)
    for rank in range(world):
        assert _oracle.rel_err(outs[rank].cpu().numpy(), ref) <= 1e-12
    assert torch.equal(outs[0], outs[1])


def test_gather_without_peers_is_contract(cuda):
    import torch
    plan, dims, sl, sr, so = _setup("zabcd,zcdef->zabef", dict(z=2, a=16, b=16, c=16, d=16, e=16, f=16),
                                    cabi.FP64)
    l = torch.rand(sl, dtype=torch.float64, device=cuda)
    r = torch.rand(sr, dtype=torch.float64, device=cuda)
    a = torch.empty(so, dtype=torch.float64, device=cuda)
    b = torch.empty(so, dtype=torch.float64, device=cuda)
    plan.contract(l, r, a)
    plan.contract_gather(l, r, b, [])
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_gather_rejects_non_contiguous_output(cuda):
    import torch
    # out rows padded to 40 columns for 32 values: not one contiguous block
    dims = [(cabi.DIM_M, 64, 64, 0, 40, 0), (cabi.DIM_N, 32, 0, 64, 1, 0), (cabi.DIM_K, 64, 1, 1, 0, 0)]
    plan = cabi.ContractPlan(dims, cabi.FP64, cabi.FP64, cabi.FP64)
    l = torch.rand(64 * 64, dtype=torch.float64, device=cuda)
    r = torch.rand(32 * 64, dtype=torch.float64, device=cuda)
    out = torch.zeros(64 * 40, dtype=torch.float64, device=cuda)
    peer = torch.zeros_like(out)
    with pytest.raises(cabi.EirError) as ei:
        plan.contract_gather(l, r, out, [peer])
    assert ei.value.code == 52
