"""eir_contract_no_alloc against eir_contract (GPU, through the C-ABI).

The no-allocation entry point exists for callers that may not call cudaMalloc
(their device memory belongs to another allocator, or the allocation's
synchronisation is not acceptable on their hot path). It must give the same
result as the allocating entry point. This file is collected last so that a
run stopping at the first failure has already run every other test, and it
works both alone in a fresh process and after the rest of the suite.
"""
import numpy as np
import pytest

from einsum_ir_b200 import binary, cabi
from tests import _oracle

pytestmark = pytest.mark.gpu

TOL = 1e-5  # relative Frobenius error, as for the BF16 contraction tests


def _plan(expr, sizes):
    il, ir, io, names = binary.parse_binary(expr)
    sz = {i: sizes[c] for i, c in enumerate(names)}
    dims = binary.contraction_dims(il, ir, io, sz)
    shapes = ([sz[i] for i in il], [sz[i] for i in ir], [sz[i] for i in io])
    return cabi.ContractPlan(dims, cabi.BF16, cabi.BF16, cabi.FP32), shapes


def test_no_alloc_matches_contract(cuda, monkeypatch):
    import torch
    monkeypatch.setenv("EIR_TC_MIN_OPS", "0")
    # BASELINE config 2 at reduced a: tensor-core path with a pre-permuted right operand
    plan, (sl, sr, so) = _plan("akmj,njk->anm", dict(a=2, k=8, m=256, j=64, n=256))
    assert plan.family == cabi.FAMILY_TC and plan.workspace_bytes > 0, plan.describe()
    g = torch.Generator().manual_seed(11)
    for call in range(2):  # two calls in a row: the shared scratch is reused
        l = ((torch.rand(sl, generator=g) * 2 - 1).to(torch.bfloat16)).to(cuda)
        r = ((torch.rand(sr, generator=g) * 2 - 1).to(torch.bfloat16)).to(cuda)
        want = torch.full(so, float("nan"), device=cuda)
        got = torch.full(so, float("nan"), device=cuda)
        plan.contract(l, r, want)
        plan.contract_no_alloc(l, r, got)
        torch.cuda.synchronize()
        err = _oracle.rel_err(got.cpu().numpy(), want.cpu().numpy())
        assert np.isfinite(got.cpu().numpy()).all()
        assert err <= TOL, f"call {call}: rel err {err:.3e}"


def test_no_alloc_split_k(cuda, monkeypatch):
    """a split-K plan: partial tiles in the static scratch, then the reduction"""
    import torch
    monkeypatch.setenv("EIR_TC_MIN_OPS", "0")
    plan, (sl, sr, so) = _plan("mk,nk->nm", dict(m=128, n=128, k=16384))
    assert "splitk=1 " not in plan.describe() and plan.workspace_bytes > 0, plan.describe()
    g = torch.Generator().manual_seed(12)
    l = ((torch.rand(sl, generator=g) * 2 - 1).to(torch.bfloat16)).to(cuda)
    r = ((torch.rand(sr, generator=g) * 2 - 1).to(torch.bfloat16)).to(cuda)
    want = torch.full(so, float("nan"), device=cuda)
    got = torch.full(so, float("nan"), device=cuda)
    plan.contract(l, r, want)
    plan.contract_no_alloc(l, r, got)
    torch.cuda.synchronize()
    assert torch.equal(got, want)  # same kernels, same slices, same summation order


def _fp64_plan():
    # BASELINE config 2's layout in FP64: the K walks disagree, so the DMMA
    # plan re-lays out the right operand (256 * 64 * 8 doubles = 1 MiB of scratch)
    il, ir, io, names = binary.parse_binary("akmj,njk->anm")
    sz = {i: dict(a=2, k=8, m=256, j=64, n=256)[c] for i, c in enumerate(names)}
    dims = binary.contraction_dims(il, ir, io, sz)
    plan = cabi.ContractPlan(dims, cabi.FP64, cabi.FP64, cabi.FP64)
    return plan, ([sz[i] for i in il], [sz[i] for i in ir], [sz[i] for i in io])


def test_no_alloc_allocates_nothing_fp64_dmma(cuda, monkeypatch):
    """On a fresh plan, eir_contract_no_alloc leaves the device's free memory
    unchanged (eir_contract would allocate the plan's workspace on its first
    call), and matches eir_contract bit for bit (same kernels)."""
    import torch
    monkeypatch.setenv("EIR_TC_MIN_OPS", "0")
    # load the library's device code and run the per-device set-up once
    warm, (sl, sr, so) = _fp64_plan()
    l = torch.rand(sl, dtype=torch.float64, device=cuda)
    r = torch.rand(sr, dtype=torch.float64, device=cuda)
    o = torch.empty(so, dtype=torch.float64, device=cuda)
    warm.contract_no_alloc(l, r, o)
    torch.cuda.synchronize()
    plan, _ = _fp64_plan()
    assert plan.family == cabi.FAMILY_DMMA and "prepack=right" in plan.describe(), plan.describe()
    assert 0 < plan.workspace_bytes <= 8 * 2 ** 20
    got = torch.full(so, float("nan"), dtype=torch.float64, device=cuda)
    want = torch.full(so, float("nan"), dtype=torch.float64, device=cuda)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(cuda)[0]
    for _ in range(2):
        plan.contract_no_alloc(l, r, got)
    torch.cuda.synchronize()
    cabi.check_device_errors()
    assert torch.cuda.mem_get_info(cuda)[0] == free0
    plan.contract(l, r, want)  # allocates the plan's own workspace on this first call
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_no_alloc_rejects_oversized_scratch(cuda):
    import torch
    # the pre-permuted (smaller) operand is the right one: 512*64*256 BF16 = 16 MiB,
    # more than the 8 MiB static scratch (left: 256*1024*64 BF16 = 32 MiB)
    plan, (sl, sr, so) = _plan("akmj,njk->anm", dict(a=1, k=256, m=1024, j=64, n=512))
    assert plan.workspace_bytes > 8 * 2 ** 20, plan.describe()
    l = torch.zeros(sl, dtype=torch.bfloat16, device=cuda)
    r = torch.zeros(sr, dtype=torch.bfloat16, device=cuda)
    out = torch.zeros(so, device=cuda)
    with pytest.raises(cabi.EirError) as ei:
        plan.contract_no_alloc(l, r, out)
    assert ei.value.code == 52 and "static scratch" in str(ei.value)
