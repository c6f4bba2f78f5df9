"""CPU tests of the oracle (test infrastructure): against torch.einsum in
float64 (the einsum semantics of at::einsum, which the reference's numeric
tests use), against the committed golden fixtures, and on the touch-kernel
and permute semantics of the reference's scalar/TPP leaves."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from einsum_ir_b200 import binary, cabi
from tests import _oracle, _tree

GOLDEN = Path(__file__).resolve().parent / "golden"


def _case(expr, sizes, seed=0, dtype=torch.float64):
    il, ir, io, names = binary.parse_binary(expr)
    sz = {i: sizes[c] for i, c in enumerate(names)}
    g = torch.Generator().manual_seed(seed)
    l = torch.rand([sz[i] for i in il], generator=g, dtype=torch.float64) * 2 - 1
    r = torch.rand([sz[i] for i in ir], generator=g, dtype=torch.float64) * 2 - 1
    return il, ir, io, sz, l.to(dtype), r.to(dtype)


@pytest.mark.parametrize("expr,sizes", [
    ("akmj,njk->anm", dict(a=2, k=3, m=5, j=4, n=6)),
    ("zabcd,zcdef->zabef", dict(z=2, a=3, b=2, c=3, d=2, e=3, f=2)),
    ("iae,cg->acegi", dict(a=2, c=3, e=2, g=3, i=2)),
    ("bf,dcba->acdf", dict(a=2, b=3, c=2, d=3, f=4)),
    ("abc,ia->bci", dict(a=3, b=4, c=5, i=6)),
])
def test_oracle_matches_torch_einsum(expr, sizes):
    il, ir, io, sz, l, r = _case(expr, sizes)
    dims = binary.contraction_dims(il, ir, io, sz)
    out = np.zeros(int(np.prod([sz[i] for i in io])))
    _oracle.contract(dims, l.numpy().ravel(), r.numpy().ravel(), out, None, cabi.FP64, cabi.FP64, cabi.FP64)
    ref = torch.einsum(expr, l, r).numpy().ravel()
    assert np.max(np.abs(out - ref)) < 1e-13


def test_oracle_bf16_and_tf32_input_rounding():
    il, ir, io, sz, l, r = _case("mk,nk->nm", dict(m=17, n=9, k=33), seed=3, dtype=torch.float32)
    dims = binary.contraction_dims(il, ir, io, sz)
    # BF16 storage: the oracle multiplies the exact BF16 values
    lb, rb = l.to(torch.bfloat16), r.to(torch.bfloat16)
    out = np.zeros(17 * 9, dtype=np.float32)
    bits = lambda t: t.view(torch.int16).numpy().view(np.uint16).ravel()
    _oracle.contract(dims, bits(lb), bits(rb), out, None, cabi.BF16, cabi.BF16, cabi.FP32)
    ref = torch.einsum("mk,nk->nm", lb.double(), rb.double()).numpy().ravel()
    assert _oracle.rel_err(out, ref) < 1e-7
    # TF32 compute: inputs rounded to nearest TF32 (ties to even) first
    x = np.array([1.0, 1.0 + 2 ** -11, 1.0 + 3 * 2 ** -11, -(1.0 + 2 ** -10 + 2 ** -12)], np.float32)
    assert list(_oracle.round_tf32(x)) == [1.0, 1.0, 1.0 + 2 ** -9, -(1.0 + 2 ** -10)]
    out_t = np.zeros(17 * 9, dtype=np.float32)
    _oracle.contract(dims, l.numpy().ravel(), r.numpy().ravel(), out_t, None, cabi.FP32, cabi.FP32,
                     cabi.FP32, cabi.COMPUTE_TF32)
    lt = torch.from_numpy(_oracle.round_tf32(l.numpy())).double()
    rt = torch.from_numpy(_oracle.round_tf32(r.numpy())).double()
    assert _oracle.rel_err(out_t, torch.einsum("mk,nk->nm", lt, rt).numpy().ravel()) < 1e-7


@pytest.mark.parametrize("first,last", [(0, 99), (3, 1), (2, 99), (99, 99), (0, 2), (3, 2)])
def test_oracle_touch_kernels(first, last):
    # semantics of ContractionBackendScalar/Tpp: first touch before the sum, last touch after
    il, ir, io, sz, l, r = _case("io,bi->bo", dict(b=5, i=7, o=6), seed=4)
    aux_sizes = {i: (1 if i == io[0] else sz[i]) for i in sz}  # bias broadcast over b
    dims = binary.contraction_dims(il, ir, io, sz, sizes_outer_aux=aux_sizes)
    rng = np.random.default_rng(0)
    out0 = rng.uniform(-1, 1, 5 * 6)
    bias = rng.uniform(-1, 1, 6)
    out = out0.copy()
    _oracle.contract(dims, l.numpy().ravel(), r.numpy().ravel(), out, bias, cabi.FP64, cabi.FP64,
                     cabi.FP64, 0, first, last)
    acc = torch.einsum("io,bi->bo", l, r).numpy()
    o0 = out0.reshape(5, 6)
    start = {0: 0.0, 3: bias[None, :], 2: o0 + bias[None, :], 99: o0}[first]
    want = start + acc
    if last == 1:
        want = np.maximum(want, 0)
    elif last == 2:
        want = want + bias[None, :]
    assert np.max(np.abs(out.reshape(5, 6) - want)) < 1e-13


def test_oracle_permute():
    rng = np.random.default_rng(1)
    x = rng.integers(0, 2 ** 31, size=(3, 4, 5, 6), dtype=np.int64).astype(np.uint32)
    perm = (2, 0, 3, 1)
    want = np.ascontiguousarray(x.transpose(perm))
    shape = list(x.shape)
    sin = [x.strides[i] // 4 for i in range(4)]
    so_perm = [want.strides[j] // 4 for j in range(4)]
    sout = [0] * 4
    for j, p in enumerate(perm):
        sout[p] = so_perm[j]
    got = np.zeros(x.size, dtype=np.uint32)
    _oracle.permute(shape, sin, sout, 4, x.ravel(), got)
    assert np.array_equal(got, want.ravel())


def _golden(name):
    f = GOLDEN / f"{name}.npz"
    return np.load(f)


@pytest.mark.parametrize("name", ["readme_tree", "readme_tree_fp64", "cfg4_tucker"])
def test_oracle_tree_matches_golden(name):
    g = _golden(name)
    n_in = len([k for k in g.files if k.startswith("in")])
    out = _tree.eval_tree(str(g["expr"]), str(g["sizes"]), str(g["path"]),
                          [g[f"in{i}"] for i in range(n_in)])
    assert _oracle.rel_err(out, g["out"]) < 1e-12


def test_oracle_binary_matches_golden():
    g = _golden("cfg2_binary_bf16")
    il, ir, io, names = binary.parse_binary(str(g["expr"]))
    sizes = [int(s) for s in str(g["sizes"]).split(",")]
    sz = {i: sizes[i] for i in range(len(names))}
    dims = binary.contraction_dims(il, ir, io, sz)
    out = np.zeros(g["out"].size, dtype=np.float32)
    _oracle.contract(dims, g["in0"].ravel(), g["in1"].ravel(), out, None, cabi.BF16, cabi.BF16, cabi.FP32)
    assert _oracle.rel_err(out, g["out"]) < 1e-6
    g = _golden("cfg5_batch_fp64")
    il, ir, io, names = binary.parse_binary(str(g["expr"]))
    sizes = [int(s) for s in str(g["sizes"]).split(",")]
    sz = {i: sizes[i] for i in range(len(names))}
    dims = binary.contraction_dims(il, ir, io, sz)
    out = np.zeros(g["out"].size)
    _oracle.contract(dims, g["in0"].ravel(), g["in1"].ravel(), out, None, cabi.FP64, cabi.FP64, cabi.FP64)
    assert _oracle.rel_err(out, g["out"]) < 1e-13


def test_oracle_mlp_layer_matches_golden():
    g = _golden("cfg3_mlp_layer")
    b, i = g["x"].shape
    o = g["w"].shape[1]
    # left = w[i][o] (M = o), right = x[b][i] (N = b): the swapped operand order of the tree
    dims = [(cabi.DIM_M, o, 1, 0, 1, 1), (cabi.DIM_N, b, 0, i, o, 0), (cabi.DIM_K, i, o, 1, 0, 0)]
    out = np.zeros(b * o, dtype=np.float32)
    _oracle.contract(dims, g["w"].ravel(), g["x"].ravel(), out, g["bias"].ravel(), cabi.FP32,
                     cabi.FP32, cabi.FP32, 0, cabi.KTYPE_COPY, cabi.KTYPE_RELU)
    assert _oracle.rel_err(out, g["out"]) < 1e-6
