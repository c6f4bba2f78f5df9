"""The etops front door (einsum_ir_b200.etops over include/eir_tensor_operation.h),
mirroring the reference's python/src/etops/__init__.py and
python/src/TensorOperation.cpp.

CPU: configuration validation and JSON form, set-up and optimize error codes,
and that `optimize` keeps the result (the oracle run on the original and on
the optimised descriptor of the same buffers). GPU: the reference README's
examples and seeded random descriptors against the oracle (FP32 within
1e-5 relative, FP64 within 1e-12).
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from einsum_ir_b200 import etops

from . import _oracle

D = etops.dim
X = etops.exec
P = etops.prim


def cfg(**kw):
    base = dict(data_type=etops.float32, prim_first=P.zero, prim_main=P.gemm, prim_last=P.none)
    base.update(kw)
    return etops.TensorOperationConfig(**base)


# ---- the reference README's examples (python/README.rst)
GEMM = cfg(backend="tpp", dim_types=(D.m, D.n, D.k), exec_types=(X.prim,) * 3, dim_sizes=(64, 32, 128),
           strides=(((1, 0, 64), (0, 128, 1), (1, 64, 0)),))
BATCHED = cfg(backend="tpp", dim_types=(D.c, D.m, D.n, D.k), exec_types=(X.shared, X.prim, X.prim, X.prim),
              dim_sizes=(48, 64, 32, 128),
              strides=(((128 * 64, 1, 0, 64), (32 * 128, 0, 128, 1), (32 * 64, 1, 64, 0)),))
PACKED = cfg(backend="tpp", dim_types=(D.m, D.n, D.k), exec_types=(X.prim,) * 3, dim_sizes=(64, 32, 128),
             strides=(((1, 0, 64), (0, 128, 1), (1, 64, 0)),
                      ((128, 0, 1), (0, 0, 0), (0, 0, 0))))
BRGEMM = cfg(dim_types=(D.k, D.m, D.n, D.k), exec_types=(X.seq,) * 4, dim_sizes=(48, 64, 32, 128),
             strides=(((128 * 64, 1, 0, 64), (32 * 128, 0, 128, 1), (0, 1, 64, 0)),))
TRANSPOSE = cfg(backend="tpp", prim_first=P.none, prim_main=P.copy, dim_types=(D.c, D.c),
                exec_types=(X.prim, X.prim), dim_sizes=(3, 4), strides=(((4, 1), (1, 3)),))
PERMUTE4 = cfg(backend="tpp", prim_first=P.none, prim_main=P.copy, dim_types=(D.c,) * 4,
               exec_types=(X.seq, X.seq, X.prim, X.prim), dim_sizes=(2, 4, 3, 5),
               strides=(((3 * 4 * 5, 5, 4 * 5, 1), (3, 2 * 3, 1, 4 * 2 * 3)),))
PERMUTE4_SEQ = cfg(prim_first=P.none, prim_main=P.copy, dim_types=(D.c,) * 4, exec_types=(X.seq,) * 4,
                   dim_sizes=(2, 4, 3, 5), strides=(((3 * 4 * 5, 5, 4 * 5, 1), (3, 2 * 3, 1, 4 * 2 * 3)),))


def _extent(c, t):
    return 1 + sum((s - 1) * max(v, 0) for s, v in zip(c.dim_sizes, c.strides[0][t]))


def _buffers(c, rng):
    binary = c.prim_main in (P.gemm, P.brgemm)
    npdt = np.float64 if c.data_type == etops.float64 else np.float32
    ins = [(rng.random(_extent(c, t)) * 2 - 1).astype(npdt) for t in range(2 if binary else 1)]
    out = (rng.random(_extent(c, 2 if binary else 1)) * 2 - 1).astype(npdt)
    return ins, out


def oracle_execute(c, ins, out):
    """the operation of configuration `c` on flat host buffers, by the CPU oracle"""
    sizes = list(c.dim_sizes)
    s = c.strides[0]
    if c.prim_main in (P.gemm, P.brgemm):
        dims = [(int(t), sz, s[0][i], s[1][i], s[2][i], 0) for i, (t, sz) in enumerate(zip(c.dim_types, sizes))]
        dt = 1 if c.data_type == etops.float64 else 0
        _oracle.contract(dims, ins[0], ins[1], out, dt_l=dt, dt_r=dt, dt_o=dt,
                         first=0 if c.prim_first == P.zero else 99,
                         last=1 if c.prim_last == P.relu else 99)
    elif c.prim_main == P.copy:
        _oracle.permute(sizes, list(s[0]), list(s[1]), out.itemsize, ins[0], out)
    else:  # zero
        offs = np.zeros(1, dtype=np.int64)
        for sz, st in zip(sizes, s[1]):
            offs = (offs[:, None] + np.arange(sz, dtype=np.int64)[None, :] * st).ravel()
        out[offs] = 0


# ------------------------------------------------------------------ CPU
BAD = [
    dict(backend="cuda"),
    dict(prim_main=P.relu),
    dict(exec_types=(X.prim,) * 2),
    dict(dim_sizes=(64, 32)),
    dict(dim_sizes=(64, 0, 128)),
    dict(strides=()),
    dict(strides=(((1, 0, 64), (0, 128, 1)),)),
    dict(strides=(((1, 0, 64), (0, 128, 1), (1, 64)),)),
    dict(prim_first=P.relu),
    dict(prim_last=P.zero),
    dict(prim_main=P.copy, prim_first=P.none, strides=(((1, 0, 64), (1, 64, 0)),)),  # unary dims must be c
    dict(prim_main=P.copy, prim_first=P.zero, dim_types=(D.c,) * 3, strides=(((1, 0, 64), (1, 64, 0)),)),
]


@pytest.mark.parametrize("kw", BAD)
def test_config_validation(kw):
    base = dict(dim_types=(D.m, D.n, D.k), exec_types=(X.prim,) * 3, dim_sizes=(64, 32, 128),
                strides=(((1, 0, 64), (0, 128, 1), (1, 64, 0)),))
    base.update(kw)
    with pytest.raises(ValueError):
        cfg(**base)


def test_json_round_trip(tmp_path):
    for c in (GEMM, PACKED, BRGEMM, PERMUTE4):
        back = etops.TensorOperationConfig.from_json(c.to_json(indent=2))
        assert back == etops.TensorOperationConfig(**{**c.__dict__, "strides": tuple(
            tuple(tuple(t) for t in lv) for lv in c.strides)})
        d = json.loads(c.to_json())
        assert d["prim_main"] in ("gemm", "copy") and d["data_type"] == "float32"
    p = tmp_path / "c.json"
    GEMM.save(str(p))
    assert etops.TensorOperationConfig.load(str(p)).to_json() == GEMM.to_json()
    with pytest.raises(ValueError):
        etops.TensorOperationConfig.from_json('{"data_type": "float32"}')
    bad = json.loads(GEMM.to_json())
    bad["prim_main"] = "gemmm"
    with pytest.raises(ValueError):
        etops.TensorOperationConfig.from_json(json.dumps(bad))


def test_setup_error_codes():
    op = etops.TensorOperation()
    E = etops.ErrorType
    dt, ex, sz = (D.m, D.n, D.k), (X.prim,) * 3, (4, 4, 4)
    ok = (((1, 0, 4), (0, 4, 1), (1, 4, 0)),)
    assert op.setup("tpp", etops.float32, P.zero, P.gemm, P.none, dt, ex, sz, ok) == E.success
    assert op.setup("tpp", etops.float32, P.zero, P.relu, P.none, dt, ex, sz, ok) == E.compilation_failed
    assert op.setup("xsmm", etops.float32, P.zero, P.gemm, P.none, dt, ex, sz, ok) == E.compilation_failed
    assert op.setup("tpp", etops.float32, P.zero, P.gemm, P.none, dt, ex, sz, ()) == E.invalid_stride_shape
    assert op.setup("tpp", etops.float32, P.zero, P.gemm, P.none, dt, ex, sz, (ok[0][:2],)) == \
        E.invalid_stride_shape
    assert op.setup("tpp", etops.float32, P.zero, P.gemm, P.none, dt, ex, sz,
                    (((1, 0), (0, 4, 1), (1, 4, 0)),)) == E.invalid_stride_shape
    un = (((1, 4), (4, 1)),)
    assert op.setup("tpp", etops.float64, P.none, P.copy, P.none, (D.c, D.c), (X.seq, X.seq), (4, 4), un) == \
        E.success
    assert op.setup("tpp", etops.float64, P.zero, P.copy, P.none, (D.c, D.c), (X.seq, X.seq), (4, 4), un) == \
        E.compilation_failed
    assert op.setup("tpp", etops.float64, P.none, P.zero, P.none, (D.c, D.c), (X.seq, X.seq), (4, 4), un) == \
        E.success
    # a failed set-up leaves nothing to execute
    assert op.setup("tpp", etops.float32, P.zero, P.brgemm, P.none, dt, ex, sz, ()) == E.invalid_stride_shape
    with pytest.raises(RuntimeError):
        op.execute(np.zeros(16, np.float32), np.zeros(16, np.float32), np.zeros(16, np.float32))
    with pytest.raises(RuntimeError):
        op.plan


def test_default_optimization_config():
    # the reference's defaults (python/src/TensorOperation.cpp:470-481)
    assert etops.backend.tpp.get_default_optimization_config() == dict(
        target_m=16, target_n=12, target_k=64, num_threads=0, br_gemm_support=True,
        packed_gemm_support=True, packing_support=True, sfc_support=True, l2_cache_size=1048576)


def test_optimize_errors():
    for bad in ({"target_q": 1}, {"target_m": "16"}, {"sfc_support": "yes"}, {"target_m": -1}):
        with pytest.raises(RuntimeError, match="invalid_optimization_config"):
            etops.optimize(BRGEMM, bad)
    r = etops.TensorOperation.optimize("tpp", etops.float32, P.zero, P.gemm, P.none, (D.m, D.n, D.k),
                                       (X.prim,) * 3, (4, 4, 4), (((1, 0, 4), (0, 4, 1)),), {})
    assert r[0] == etops.ErrorType.invalid_stride_shape and list(r[8]) == []
    r = etops.TensorOperation.optimize("tpp", etops.float32, P.zero, P.none, P.none, (D.m, D.n, D.k),
                                       (X.prim,) * 3, (4, 4, 4), (((1, 0, 4), (0, 4, 1), (1, 4, 0)),), {})
    assert r[0] == etops.ErrorType.compilation_failed
    assert BRGEMM.backend is None and etops.optimize(BRGEMM).backend == "tpp"


def _random_binary(rng, fp64):
    """a random binary descriptor: every tensor dense in a random dim order"""
    nd = int(rng.integers(3, 7))
    types = [D.m, D.n, D.k] + [etops.DimType(int(t)) for t in rng.integers(0, 4, nd - 3)]
    rng.shuffle(types)
    sizes = [int(x) for x in rng.integers(1, 9, nd)]
    dims_of = {0: [i for i, t in enumerate(types) if t in (D.c, D.m, D.k)],
               1: [i for i, t in enumerate(types) if t in (D.c, D.n, D.k)],
               2: [i for i, t in enumerate(types) if t in (D.c, D.m, D.n)]}
    strides = []
    for t in range(3):
        order = list(rng.permutation(dims_of[t]))
        st, acc = [0] * nd, 1
        for i in reversed(order):
            st[i] = acc
            acc *= sizes[i]
        strides.append(tuple(st))
    return cfg(data_type=etops.float64 if fp64 else etops.float32,
               prim_first=P.zero if rng.random() < 0.6 else P.none,
               prim_last=P.relu if rng.random() < 0.3 else P.none,
               prim_main=P.gemm if rng.random() < 0.5 else P.brgemm,
               dim_types=tuple(types), exec_types=tuple(etops.ExecType(int(e)) for e in rng.integers(0, 4, nd)),
               dim_sizes=tuple(sizes), strides=(tuple(strides),))


def _random_unary(rng, zero):
    nd = int(rng.integers(1, 6))
    sizes = [int(x) for x in rng.integers(1, 7, nd)]
    strides = []
    for _ in range(2):
        order = list(rng.permutation(nd))
        st, acc = [0] * nd, 1
        for i in reversed(order):
            st[i] = acc
            acc *= sizes[i]
        strides.append(tuple(st))
    return cfg(prim_first=P.none, prim_main=P.zero if zero else P.copy, dim_types=(D.c,) * nd,
               exec_types=(X.seq,) * nd, dim_sizes=tuple(sizes), strides=(tuple(strides),))


@pytest.mark.parametrize("seed", range(12))
def test_optimize_keeps_the_result(seed):
    rng = np.random.default_rng(seed)
    cases = [_random_binary(rng, seed % 2 == 1), _random_unary(rng, False), _random_unary(rng, True)]
    if seed == 0:
        cases += [GEMM, BATCHED, PACKED, BRGEMM, TRANSPOSE, PERMUTE4, PERMUTE4_SEQ]
    for c in cases:
        o = etops.optimize(c)
        assert len(o.dim_sizes) <= len(c.dim_sizes) and len(o.strides) == 1
        assert np.prod(o.dim_sizes) == np.prod(c.dim_sizes)
        ins, out = _buffers(c, rng)
        out2 = out.copy()
        oracle_execute(c, ins, out)
        oracle_execute(o, ins, out2)
        tol = 1e-12 if c.data_type == etops.float64 else 1e-5
        assert _oracle.rel_err(out2, out) <= tol, (c, o)
        etops.TensorOperation(o)  # the optimised descriptor sets up


def test_execute_checks_extents():
    op = etops.TensorOperation(GEMM)
    a, b = np.zeros(128 * 64, np.float32), np.zeros(32 * 128, np.float32)
    with pytest.raises(ValueError, match="in0"):
        op.execute(a[:-1], b, np.zeros(32 * 64, np.float32))
    with pytest.raises(ValueError, match="out"):
        op.execute(a, b, np.zeros(32 * 64 - 1, np.float32))
    with pytest.raises(ValueError):
        op.execute(a, b, np.zeros(32 * 64, np.float64))
    with pytest.raises(ValueError):
        op.execute(a, None, np.zeros(32 * 64, np.float32))
    neg = cfg(dim_types=(D.m, D.n, D.k), exec_types=(X.prim,) * 3, dim_sizes=(4, 4, 4),
              strides=(((-1, 0, 4), (0, 4, 1), (1, 4, 0)),))
    with pytest.raises(ValueError, match="in0"):
        etops.TensorOperation(neg).execute(np.zeros(64, np.float32), np.zeros(64, np.float32),
                                           np.zeros(64, np.float32))


# ------------------------------------------------------------------ GPU
def _gpu_check(c, rng, kind="numpy"):
    import torch
    ins, out = _buffers(c, rng)
    want = out.copy()
    oracle_execute(c, ins, want)
    op = etops.TensorOperation(c)
    if kind == "numpy":
        got = out.copy()
        op.execute(ins[0], ins[1] if len(ins) > 1 else None, got)
    elif kind == "torch_cpu":
        t = torch.from_numpy(out.copy())
        op.execute(torch.from_numpy(ins[0]), torch.from_numpy(ins[1]) if len(ins) > 1 else None, t)
        got = t.numpy()
    else:
        dev = torch.device("cuda:0")
        t = torch.from_numpy(out.copy()).to(dev)
        op.execute(torch.from_numpy(ins[0]).to(dev), torch.from_numpy(ins[1]).to(dev) if len(ins) > 1 else None, t)
        torch.cuda.synchronize()
        got = t.cpu().numpy()
    from einsum_ir_b200 import cabi
    cabi.check_device_errors()
    tol = 1e-12 if c.data_type == etops.float64 else 1e-5
    err = _oracle.rel_err(got, want)
    assert err <= tol, f"{err:.3e} | {op.describe()} | {c}"
    return op


@pytest.mark.gpu
@pytest.mark.parametrize("name,c,kind", [
    ("transpose", TRANSPOSE, "numpy"), ("permute4", PERMUTE4, "numpy"),
    ("permute4_optimized", None, "numpy"), ("gemm", GEMM, "numpy"), ("batched", BATCHED, "torch_cpu"),
    ("packed", PACKED, "numpy"), ("brgemm_optimized", None, "torch_cpu"), ("gemm_device", GEMM, "cuda")])
def test_reference_readme_examples(cuda, name, c, kind):
    if name == "permute4_optimized":
        c = etops.optimize(PERMUTE4_SEQ)
    if name == "brgemm_optimized":
        c = etops.optimize(BRGEMM, {"target_m": 16, "target_n": 12, "target_k": 64, "num_threads": 4,
                                    "br_gemm_support": True, "packed_gemm_support": True})
    _gpu_check(c, np.random.default_rng(3), kind)


@pytest.mark.gpu
@pytest.mark.parametrize("seed", range(16))
def test_random_descriptors(cuda, seed):
    rng = np.random.default_rng(100 + seed)
    _gpu_check(_random_binary(rng, seed % 2 == 1), rng, "cuda")
    _gpu_check(_random_unary(rng, False), rng, "cuda")
    _gpu_check(_random_unary(rng, True), rng, "numpy")


@pytest.mark.gpu
@pytest.mark.parametrize("fp64", [False, True])
@pytest.mark.parametrize("first,last", [(P.zero, P.none), (P.none, P.relu)])
def test_tensor_core_sizes(cuda, fp64, first, last):
    """a contraction big enough for the tensor-core kernels (3xTF32 / DMMA):
    C x K-major M x MN-major N over two K dims"""
    from einsum_ir_b200 import cabi
    c, m, n, k1, k2 = 2, 256, 192, 16, 16
    k = k1 * k2
    c_ = cfg(data_type=etops.float64 if fp64 else etops.float32, prim_first=first, prim_last=last,
             dim_types=(D.c, D.m, D.n, D.k, D.k), exec_types=(X.shared, X.prim, X.prim, X.seq, X.prim),
             dim_sizes=(c, m, n, k1, k2),
             strides=(((m * k, k, 0, k2, 1), (k * n, 0, 1, k2 * n, n), (m * n, 1, m, 0, 0)),))
    op = _gpu_check(c_, np.random.default_rng(7), "cuda")
    assert op.plan.family in (cabi.FAMILY_TC, cabi.FAMILY_DMMA), op.describe()
