"""CPU tests that pin the C oracle's numerics to the reference itself.

The reference's own scalar contraction backend (backend::BinaryContractionScalar
over basic::ContractionBackend, src/backend/BinaryContractionScalar.cpp:4-144,
src/basic/binary/ContractionBackend.cpp:251-515, ContractionBackendScalar.cpp:4-142)
and its scalar permute (backend::UnaryScalar) are compiled from the reference
sources into oracle/_ref/libref_scalar.so (oracle/ref.mk, with a stand-in for
the absent libxsmm header). Here they run on the same seeded inputs as the C
oracle (oracle/eir_oracle.c): the golden shapes, the BASELINE configs at
reduced sizes, random dim orders, every first/last-touch kernel with
broadcast bias, FP32 and FP64, and the committed golden fixtures. Skipped when
the reference library was not built (no reference checkout at build time)."""
from __future__ import annotations

import random
from pathlib import Path

import numpy as np
import pytest

from einsum_ir_b200 import binary, cabi
from tests import _oracle, _refscalar

pytestmark = pytest.mark.skipif(not _refscalar.available(),
                                reason="reference scalar library not built (needs the reference sources)")

GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = {cabi.FP64: 1e-12, cabi.FP32: 1e-5}  # relative Frobenius (FP32: the reference sums in FP32)


def _both(expr_or_ids, sizes, dtype, first=cabi.KTYPE_ZERO, last=cabi.KTYPE_UNDEFINED,
          aux_bcast=(), seed=0):
    """(oracle result, reference result, reference num_ops) on the same inputs."""
    if isinstance(expr_or_ids, str):
        il, ir, io, names = binary.parse_binary(expr_or_ids)
        sz = {i: sizes[c] for i, c in enumerate(names)}
    else:
        il, ir, io = expr_or_ids
        sz = dict(sizes)
    npdt = np.float64 if dtype == cabi.FP64 else np.float32
    rng = np.random.default_rng(seed)
    shp = lambda ids: [sz[i] for i in ids]
    l = rng.uniform(-1, 1, shp(il)).astype(npdt)
    r = rng.uniform(-1, 1, shp(ir)).astype(npdt)
    out0 = rng.uniform(-1, 1, shp(io)).astype(npdt)
    uses_aux = first in (cabi.KTYPE_COPY, cabi.KTYPE_ADD) or last == cabi.KTYPE_ADD
    aux_outer = {i: (1 if i in aux_bcast else sz[i]) for i in sz} if uses_aux else None
    aux = rng.uniform(-1, 1, [aux_outer[i] for i in io]).astype(npdt) if uses_aux else None
    dims = binary.contraction_dims(il, ir, io, sz, sizes_outer_aux=aux_outer)
    got = out0.copy()
    _oracle.contract(dims, l.ravel(), r.ravel(), got.ravel(), None if aux is None else aux.ravel(),
                     dtype, dtype, dtype, 0, first, last)
    ref = out0.copy()
    try:
        rc = _refscalar.Contraction(il, ir, io, sz, dtype=dtype, first=first, last=last,
                                    aux_outer=aux_outer, threads=1)
    except RuntimeError as e:  # the reference's own compile rejects the case
        pytest.skip(str(e))
    rc.contract(l, r, ref, aux)
    return got, ref, rc.num_ops, dims


@pytest.mark.parametrize("dtype", [cabi.FP32, cabi.FP64])
@pytest.mark.parametrize("expr,sizes", [
    # the README expression's contractions at the reference test's sizes
    # (EinsumExpression.test.torch.cpp:695) and BASELINE configs 2-5 reduced
    ("bf,dcba->acdf", dict(a=8, b=4, c=2, d=16, f=8)),
    ("dh,acdf->acfh", dict(a=8, c=2, d=16, f=8, h=8)),
    ("iae,cg->acegi", dict(a=8, c=2, e=6, g=4, i=8)),
    ("acfh,acegi->hgfei", dict(a=4, c=2, e=3, f=4, g=2, h=3, i=4)),
    ("akmj,njk->anm", dict(a=2, k=3, m=7, j=5, n=6)),
    ("bi,io->bo", dict(b=9, i=13, o=7)),
    ("abc,ia->bci", dict(a=5, b=4, c=3, i=6)),
    ("zabcd,zcdef->zabef", dict(z=3, a=2, b=3, c=4, d=2, e=3, f=2)),
])
def test_oracle_equals_reference_scalar(expr, sizes, dtype):
    got, ref, ops, dims = _both(expr, sizes, dtype)
    assert _oracle.rel_err(got, ref) <= TOL[dtype]
    # the reference's flop count (BinaryContraction.cpp:434-465) is this backend's
    assert ops == cabi.ContractPlan(dims, dtype, dtype, dtype).num_ops


# the scalar backend implements first touch ZERO / COPY and last touch RELU
# (ContractionBackendScalar.cpp:70-115); ADD exists only in the libxsmm
# backend, whose semantics the oracle restates (ContractionBackendTpp.cpp:130-163)
SCALAR_TOUCHES = [(cabi.KTYPE_ZERO, cabi.KTYPE_RELU), (cabi.KTYPE_COPY, cabi.KTYPE_UNDEFINED),
                  (cabi.KTYPE_COPY, cabi.KTYPE_RELU), (cabi.KTYPE_UNDEFINED, cabi.KTYPE_UNDEFINED),
                  (cabi.KTYPE_UNDEFINED, cabi.KTYPE_RELU), (cabi.KTYPE_ZERO, cabi.KTYPE_UNDEFINED)]


@pytest.mark.parametrize("dtype", [cabi.FP32, cabi.FP64])
@pytest.mark.parametrize("first,last", SCALAR_TOUCHES)
def test_touch_kernels_equal_reference(first, last, dtype):
    # bias broadcast over the batch dim b (the MLP layer of bench_mlp.cpp:207-290)
    il, ir, io, names = binary.parse_binary("io,bi->bo")
    sz = {i: s for i, s in zip(range(3), (11, 13, 7))}  # b, i, o
    got, ref, _, _ = _both((il, ir, io), sz, dtype, first, last, aux_bcast=(io[0],), seed=5)
    assert _oracle.rel_err(got, ref) <= TOL[dtype]


def _random_ids(rng: random.Random):
    """random C/M/N/K dims, each tensor in a random dim order"""
    n = {t: rng.randint(lo, 2) for t, lo in (("c", 0), ("m", 1), ("n", 1), ("k", 1))}
    ids, i = {}, 0
    for t in "cmnk":
        ids[t] = list(range(i, i + n[t]))
        i += n[t]
    il = ids["c"] + ids["m"] + ids["k"]
    ir = ids["c"] + ids["n"] + ids["k"]
    io = ids["c"] + ids["m"] + ids["n"]
    for x in (il, ir, io):
        rng.shuffle(x)
    # the reference's optimizer rejects (COMPILATION_FAILED) an output whose
    # unit-stride dim is a C dim; the C oracle and this backend accept it
    while io[-1] in ids["c"]:
        io.insert(0, io.pop())
    sizes = {d: rng.randint(1 if rng.random() < 0.5 else 2, 5) for d in range(i)}
    return (il, ir, io), sizes, ids


@pytest.mark.parametrize("seed", range(32))
def test_random_dim_orders_equal_reference(seed):
    rng = random.Random(seed)
    ids3, sizes, groups = _random_ids(rng)
    dtype = cabi.FP64 if seed % 2 else cabi.FP32
    first, last = rng.choice(SCALAR_TOUCHES)
    bcast = tuple(d for d in groups["c"] + groups["m"] + groups["n"] if rng.random() < 0.3)
    got, ref, _, _ = _both(ids3, sizes, dtype, first, last, aux_bcast=bcast, seed=seed)
    assert _oracle.rel_err(got, ref) <= TOL[dtype]


@pytest.mark.parametrize("seed", range(8))
def test_permute_equals_reference_unary(seed):
    rng = random.Random(100 + seed)
    nd = rng.randint(1, 5)
    ids_in = list(range(nd))
    ids_out = ids_in[:]
    rng.shuffle(ids_out)
    sizes = {d: rng.randint(1, 6) for d in ids_in}
    dtype = cabi.FP64 if seed % 2 else cabi.FP32
    npdt = np.float64 if dtype == cabi.FP64 else np.float32
    src = np.random.default_rng(seed).uniform(-1, 1, [sizes[d] for d in ids_in]).astype(npdt)
    ref = np.zeros([sizes[d] for d in ids_out], dtype=npdt)
    _refscalar.permute(ids_in, ids_out, sizes, src, ref, dtype)
    sin = binary.strides(ids_in, sizes)
    sout = binary.strides(ids_out, sizes)
    got = np.zeros_like(ref)
    _oracle.permute([sizes[d] for d in ids_in], [sin[d] for d in ids_in], [sout[d] for d in ids_in],
                    src.itemsize, src.ravel(), got.ravel())
    assert np.array_equal(got, ref)


def _ref_binary(expr, l, r):
    """one contraction through the reference's scalar backend (FP64, ZERO first touch)"""
    il, ir, io, names = binary.parse_binary(expr)
    sz = {}
    for ids, t in ((il, l), (ir, r)):
        for i, s in zip(ids, t.shape):
            sz[i] = s
    out = np.zeros([sz[i] for i in io])
    c = _refscalar.Contraction(il, ir, io, sz, dtype=cabi.FP64, first=cabi.KTYPE_ZERO, threads=1)
    c.contract(np.ascontiguousarray(l, np.float64), np.ascontiguousarray(r, np.float64), out)
    return out


def test_golden_fixtures_equal_reference():
    """the committed golden outputs (torch.einsum in float64) equal the
    reference's own scalar backend run on the fixtures' inputs"""
    d = np.load(GOLDEN / "cfg5_batch_fp64.npz", allow_pickle=False)
    assert _oracle.rel_err(_ref_binary("zabcd,zcdef->zabef", d["in0"], d["in1"]), d["out"]) <= 1e-12
    # Tucker abc,ia,jb,kc->ijk, one binary step at a time
    d = np.load(GOLDEN / "cfg4_tucker.npz", allow_pickle=False)
    t = _ref_binary("abc,ia->bci", d["in0"], d["in1"])
    t = _ref_binary("bci,jb->cij", t, d["in2"])
    t = _ref_binary("cij,kc->ijk", t, d["in3"])
    assert _oracle.rel_err(t, d["out"]) <= 1e-12


def test_readme_tree_fixture_equals_reference():
    """the README expression iae,bf,dcba,cg,dh->hgfei (path (1,2),(2,3),(0,1),(0,1))
    evaluated binary step by step through the reference's scalar backend, with
    the intermediates its tree rules give (dims in ascending id order:
    EinsumExpression.cpp:25-99), equals the committed FP64 golden output"""
    d = np.load(GOLDEN / "readme_tree_fp64.npz", allow_pickle=False)
    acdf = _ref_binary("bf,dcba->acdf", d["in1"], d["in2"])
    acfh = _ref_binary("dh,acdf->acfh", d["in4"], acdf)
    acegi = _ref_binary("iae,cg->acegi", d["in0"], d["in3"])
    out = _ref_binary("acfh,acegi->hgfei", acfh, acegi)
    assert _oracle.rel_err(out, d["out"]) <= 1e-12


def test_mlp_layer_fixture_equals_reference():
    """one bench_mlp hidden layer, relu(x w + bias), through the reference's
    scalar backend: COPY first touch of the bias broadcast over b (outer size
    1, so stride 0), MADD, RELU last touch (ContractionBackendScalar.cpp:70-115),
    on the fixture's inputs in FP64, equals the committed golden output"""
    d = np.load(GOLDEN / "cfg3_mlp_layer.npz", allow_pickle=False)
    x, w, bias = (d[k].astype(np.float64) for k in ("x", "w", "bias"))
    il, ir, io, names = binary.parse_binary("bi,io->bo")
    sz = {i: n for i, n in zip(range(3), (x.shape[0], x.shape[1], w.shape[1]))}  # b, i, o
    aux_outer = {i: (1 if names[i] == "b" else sz[i]) for i in sz}
    out = np.zeros([sz[i] for i in io])
    c = _refscalar.Contraction(il, ir, io, sz, dtype=cabi.FP64, first=cabi.KTYPE_COPY, last=cabi.KTYPE_RELU,
                               aux_outer=aux_outer, threads=1)
    c.contract(np.ascontiguousarray(x), np.ascontiguousarray(w), out, bias.reshape(1, -1).copy())
    assert _oracle.rel_err(out, d["out"]) <= 1e-12


@pytest.mark.parametrize("dtype", [cabi.FP32, cabi.FP64])
def test_long_k_equals_reference(dtype):
    """K = 6144 over two K dims: the reference's scalar backend sums in the
    data type (an FP32 running sum for FP32), the oracle in FP64 / long double;
    they agree to the FP32 tolerance"""
    got, ref, _, _ = _both("mkq,nqk->nm", dict(m=5, n=6, k=1024, q=6), dtype, seed=9)
    assert _oracle.rel_err(got, ref) <= TOL[dtype]


def test_bf16_fixture_equals_reference_fp64():
    """config 2 (akmj,njk->anm) has BF16 inputs, which the reference cannot
    read; every BF16 value is exact in FP64, so the reference's FP64 scalar
    backend on the fixture's inputs gives the exact products the golden
    output holds"""
    d = np.load(GOLDEN / "cfg2_binary_bf16.npz", allow_pickle=False)
    as_f64 = lambda u: (u.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    out = _ref_binary("akmj,njk->anm", as_f64(d["in0"]), as_f64(d["in1"]))
    assert _oracle.rel_err(out, d["out"]) <= 1e-12
