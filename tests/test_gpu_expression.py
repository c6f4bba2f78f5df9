"""GPU parity of einsum trees through the C-ABI expression entry points
(EinsumExpression -> EinsumNode tree -> CUDA contractions), mirroring the
reference's EinsumExpression.test.torch.cpp:695-787 (the README expression,
its sizes and path) and the BASELINE configs at reduced sizes, against the
committed golden fixtures and the CPU oracle."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from einsum_ir_b200 import binary, cabi
from tests import _oracle, _tree

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _run_expression(cuda, g, dtype, comp=cabi.COMPUTE_DEFAULT, stream=None, repeats=1):
    import torch
    expr = cabi.Expression(str(g["expr"]), str(g["sizes"]), str(g["path"]), dtype, comp)
    n_in = expr.num_tensors - 1
    ins = []
    for i in range(n_in):
        a = g[f"in{i}"]
        t = torch.from_numpy(a.view(np.int16)).view(torch.bfloat16) if a.dtype == np.uint16 else torch.from_numpy(a)
        assert list(t.shape) == expr.tensor_shape(i)
        ins.append(t.to(cuda))
    odt = torch.float64 if dtype == cabi.FP64 else torch.float32
    out = torch.full(expr.tensor_shape(n_in), float("nan"), dtype=odt, device=cuda)
    sp = 0 if stream is None else stream.cuda_stream
    results = []
    for _ in range(repeats):
        out.fill_(float("nan"))
        expr.eval(ins + [out], stream=sp)
        torch.cuda.synchronize()
        results.append(out.cpu().numpy().copy())
    cabi.check_device_errors()
    return expr, results


@pytest.mark.parametrize("name,dtype,tol", [
    ("readme_tree", cabi.FP32, 1e-5),
    ("readme_tree_fp64", cabi.FP64, 1e-12),
    ("cfg4_tucker", cabi.FP32, 1e-5),
    ("cfg2_binary_bf16", cabi.BF16, 1e-5),
    ("cfg5_batch_fp64", cabi.FP64, 1e-12),
])
def test_expression_matches_golden(cuda, name, dtype, tol):
    g = np.load(GOLDEN / f"{name}.npz")
    expr, (got,) = _run_expression(cuda, g, dtype)
    err = _oracle.rel_err(got, g["out"])
    assert np.isfinite(got).all()
    assert err <= tol, f"{name}: rel err {err:.3e}\n{expr.describe()}"


def test_expression_graph_replay(cuda):
    import torch
    g = np.load(GOLDEN / "readme_tree.npz")
    s = torch.cuda.Stream()
    expr, results = _run_expression(cuda, g, cabi.FP32, stream=s, repeats=4)  # eager, capture, replay x2
    for r in results:
        assert _oracle.rel_err(r, g["out"]) <= 1e-5


def test_readme_config_full_size(cuda):
    import torch
    expr_s, sizes, path = "iae,bf,dcba,cg,dh->hgfei", "32,8,4,2,16,64,8,8,8", "(1,2),(2,3),(0,1),(0,1)"
    expr = cabi.Expression(expr_s, sizes, path, cabi.FP32)
    assert expr.num_ops == 134742016 or expr.num_ops > 1.3e8
    gen = torch.Generator().manual_seed(0)
    ins = [torch.rand(expr.tensor_shape(i), generator=gen) * 2 - 1 for i in range(5)]
    out = torch.zeros(expr.tensor_shape(5), device=cuda)
    expr.eval([t.to(cuda) for t in ins] + [out])
    torch.cuda.synchronize()
    ref = _tree.eval_tree(expr_s, sizes, path, [t.numpy() for t in ins])
    err = _oracle.rel_err(out.cpu().numpy(), ref)
    assert err <= 1e-5, f"{err:.3e}\n{expr.describe()}"


@pytest.mark.parametrize("dtype", ["fp32", "tf32", "bf16"])
def test_mlp_chain_bias_relu(cuda, dtype, monkeypatch):
    """4 layers of bench_mlp's node pattern (COPY bias first touch, MADD, RELU last
    touch on the hidden layers, bias only on the last) at reduced sizes."""
    import torch
    monkeypatch.setenv("EIR_TC_MIN_OPS", "0")
    b, w = 256, 192
    gen = torch.Generator().manual_seed(3)
    x = torch.rand(b, w, generator=gen, dtype=torch.float64) * 2 - 1
    ws = [torch.randn(w, w, generator=gen, dtype=torch.float64) / w ** 0.5 for _ in range(4)]
    bs = [torch.rand(w, generator=gen, dtype=torch.float64) * 2 - 1 for _ in range(4)]
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    if dtype == "tf32":
        rnd = lambda t: torch.from_numpy(_oracle.round_tf32(t.float().numpy())).double()
        ws = [rnd(m) for m in ws]
    # reference: fp64 on the inputs rounded to the compute type
    h_ref = x.to(tdt).double()
    act = x.to(tdt).to(cuda)
    for layer in range(4):
        wl = ws[layer].to(tdt)
        # left = weight[i][o] (M = o), right = activation[b][i] (N = b), out[b][o]
        dims = [(cabi.DIM_M, w, 1, 0, 1, 1), (cabi.DIM_N, b, 0, w, w, 0), (cabi.DIM_K, w, w, 1, 0, 0)]
        last = cabi.KTYPE_RELU if layer < 3 else cabi.KTYPE_UNDEFINED
        dl = cabi.BF16 if dtype == "bf16" and layer == 0 else cabi.FP32
        dw = cabi.BF16 if dtype == "bf16" else cabi.FP32
        comp = cabi.COMPUTE_TF32 if dtype == "tf32" else cabi.COMPUTE_DEFAULT
        if dtype == "bf16" and dl != dw:
            act = act.to(torch.bfloat16)
            dl = cabi.BF16
        plan = cabi.ContractPlan(dims, dw, dl, cabi.FP32, comp, cabi.KTYPE_COPY, cabi.KTYPE_MADD, last)
        out = torch.empty(b, w, device=cuda)
        plan.contract(wl.to(cuda), act, out, aux=bs[layer].float().to(cuda))
        h_ref = h_ref @ wl.double() + bs[layer].float().double()
        if layer < 3:
            h_ref = torch.relu(h_ref)
        act = out.to(torch.bfloat16) if dtype == "bf16" else out
        h_ref = h_ref.to(tdt).double() if dtype == "bf16" else h_ref
    torch.cuda.synchronize()
    err = _oracle.rel_err(act.float().cpu().numpy(), h_ref.numpy())
    tol = {"fp32": 1e-5, "tf32": 5e-3, "bf16": 1e-2}[dtype]
    assert err <= tol, f"{dtype}: {err:.3e}"
