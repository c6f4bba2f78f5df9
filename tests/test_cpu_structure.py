"""CPU tests of the host logic: the reference's structural known answers, a
differential check of the host layer against the reference's own structural
functions (compiled from its sources into oracle/_ref), the C-ABI exports and
the planner's lowering decisions (no GPU needed)."""
from __future__ import annotations

import ctypes
import random
import re
import subprocess
from pathlib import Path

import pytest

from einsum_ir_b200 import binary, cabi

ROOT = Path(__file__).resolve().parents[1]
HOST = ROOT / "einsum_ir_b200" / "host_unit_tests"
REFLIB = ROOT / "oracle" / "_ref" / "libref_struct.so"


def _header_functions():
    """every function declared by the C-ABI headers under include/"""
    names = set()
    for h in sorted((ROOT / "include").glob("*.h")):
        txt = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(eir_[a-z0-9_]+)\s*\(", txt))
    return sorted(names)


def test_host_unit_tests():
    r = subprocess.run([str(HOST)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def test_library_exports_every_declared_symbol():
    lib = cabi.lib()
    names = _header_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(cabi.EXPORTS) == set(names)


def _ref():
    if not REFLIB.exists():
        pytest.skip("reference structural library not built (needs the reference sources)")
    L = ctypes.CDLL(str(REFLIB))
    return L


def _host(lines):
    r = subprocess.run([str(HOST), "--cases"], input="\n".join(lines) + "\n", capture_output=True,
                       text=True, check=True)
    return r.stdout.rstrip("\n").split("\n")


def _random_case(rng):
    n = rng.randint(1, 8)
    dims = list(range(n))
    pick = lambda: [d for d in dims if rng.random() < 0.6]
    l, r = pick(), pick()
    o = [d for d in dims if (d in l) != (d in r) or (rng.random() < 0.5 and d in l and d in r)]
    for x in (l, r, o):
        rng.shuffle(x)
    return l or [0], r or [0], o


def _arr(v):
    return (ctypes.c_int64 * max(1, len(v)))(*v)


def test_dim_types_and_swap_match_reference():
    L = _ref()
    rng = random.Random(0)
    cases = [_random_case(rng) for _ in range(300)]
    lines_t = [f"T {len(l)} {len(r)} {len(o)} " + " ".join(map(str, l + r + o)) for l, r, o in cases]
    lines_s = [f"S {len(l)} {len(r)} {len(o)} " + " ".join(map(str, l + r + o)) for l, r, o in cases]
    host_t, host_s = _host(lines_t), _host(lines_s)
    for (l, r, o), ht, hs in zip(cases, host_t, host_s):
        tl, tr, to = (ctypes.c_int32 * max(1, len(l)))(), (ctypes.c_int32 * max(1, len(r)))(), \
            (ctypes.c_int32 * max(1, len(o)))()
        L.ref_dim_types(len(l), len(r), len(o), _arr(l), _arr(r), _arr(o), tl, tr, to)
        ref_types = list(tl[:len(l)]) + list(tr[:len(r)]) + list(to[:len(o)])
        assert [int(x) for x in ht.split()] == ref_types, (l, r, o)
        py = binary.dim_types(l, r, o)
        assert py[0] + py[1] + py[2] == ref_types
        ref_swap = L.ref_swap_inputs(len(l), len(r), len(o), _arr(l), _arr(r), _arr(o))
        assert int(hs) == ref_swap, (l, r, o)
        assert int(binary.swap_inputs(l, r, o)) == ref_swap


def test_expression_helpers_match_reference():
    L = _ref()
    rng = random.Random(1)
    for _ in range(100):
        n = rng.randint(1, 6)
        path = []
        for c in range(n):
            live = n + 1 - c
            a, b = rng.sample(range(live), 2)
            path += [a, b]
        out = (ctypes.c_int64 * (2 * n))()
        L.ref_unique_tensor_ids(n, _arr(path), out)
        host = _host([f"U {n} " + " ".join(map(str, path))])[0]
        assert [int(x) for x in host.split()] == list(out)
    for _ in range(100):
        nh = rng.randint(2, 9)
        l = rng.sample(range(nh), rng.randint(1, nh))
        r = rng.sample(range(nh), rng.randint(1, nh))
        hist = [rng.randint(0, 3) for _ in range(nh)]
        for d in l + r:
            hist[d] += 1
        h_ref = _arr(hist)
        out = (ctypes.c_int64 * 16)()
        k = L.ref_substring_out(len(l), len(r), _arr(l), _arr(r), h_ref, out, 16)
        host = _host([f"B {len(l)} {len(r)} {nh} " + " ".join(map(str, l + r + hist))])[0]
        assert [int(x) for x in host.split()] == list(out[:k])


def test_parse_dim_ids_match_reference():
    L = _ref()
    exprs = ["[i,aaa,e],[b,f],[d,c,b,aaa],[c,g],[d,h]->[h,g,f,e,i]",
             "[13,5,9],[6,10],[8,7,6,5],[7,11],[8,12]->[12,11,10,9,13]",
             "[x1,y,2],[2,x1]->[y]", "[a,b],[b,c]->[a,c]"]
    host = _host([f"D {e}" for e in exprs])
    for e, h in zip(exprs, host):
        buf = ctypes.create_string_buffer(4096)
        L.ref_parse_dim_ids(e.encode(), buf, 4096)
        assert buf.value.decode() == h


def _random_tree(rng, depth=0):
    """A random einsum tree string (leaves, permutes, binary nodes) and its root dims."""
    r = rng.random()
    if depth >= 3 or r < 0.3:
        ids = rng.sample(range(14), rng.randint(1, 4))
        return ",".join(map(str, ids)), ids
    if r < 0.45:
        s, ids = _random_tree(rng, depth + 1)
        out = ids[:]
        rng.shuffle(out)
        return f"[{s}]->[{','.join(map(str, out))}]", out
    (sl, il), (sr, ir) = _random_tree(rng, depth + 1), _random_tree(rng, depth + 1)
    both = list(dict.fromkeys(il + ir))
    out = [d for d in both if rng.random() < 0.7] or both[:1]
    rng.shuffle(out)
    return f"[{sl}],[{sr}]->[{','.join(map(str, out))}]", out


def test_tree_parser_matches_reference():
    L = _ref()
    rng = random.Random(3)
    trees = ["[[3,0]->[0,3]],[[3,2,4],[1,4,2]->[1,2,3]]->[0,1,2]", "[0,3],[1,2,3]->[0,1,2]",
             "[0,1]->[1,0]"] + [_random_tree(rng)[0] for _ in range(150)]
    trees = [t for t in trees if t.startswith("[")]
    lines = []
    for t in trees:
        n_ids = len(set(int(x) for x in re.findall(r"\d+", t)))
        lines.append((t, ",".join(str(2 + i) for i in range(n_ids))))
    host = _host([f"E {t} {sz}" for t, sz in lines])
    for (t, sz), h in zip(lines, host):
        buf = ctypes.create_string_buffer(1 << 16)
        k = L.ref_parse_tree(t.encode(), sz.encode(), buf, 1 << 16)
        assert (buf.value.decode() if k >= 0 else "-1") == h, t


PLAN_CASES = [
    # expression, sizes, dtype, compute, expected lowering fragments
    ("akmj,njk->anm", dict(a=16, k=32, m=512, j=64, n=512), cabi.BF16, 0,
     ["tc kind=bf16", "BN=256", "prepack=right"]),
    ("zcdef,zabcd->zabef", dict(z=64, a=48, b=48, c=48, d=48, e=48, f=48), cabi.FP32,
     cabi.COMPUTE_TF32, ["tc kind=tf32", "A=MN B=K", "M=2304 N=2304 Kp=2304"]),
    ("io,bi->bo", dict(b=8192, i=4096, o=4096), cabi.FP32, 0, ["tc kind=3xtf32", "A=MN B=K"]),
    ("io,bi->bo", dict(b=8192, i=4096, o=4096), cabi.BF16, 0, ["tc kind=bf16", "A=MN B=K"]),
    ("zcdef,zabcd->zabef", dict(z=64, a=48, b=48, c=48, d=48, e=48, f=48), cabi.FP64, 0,
     ["tc kind=fp64-dmma", "A=MN B=K"]),
    ("acfh,acegi->hgfei", dict(a=32, c=4, e=16, f=64, g=8, h=8, i=8), cabi.FP32, 0, ["simt"]),
    # the README tree's first step: tiny, one output element per thread
    ("dcba,bf->facd", dict(a=32, b=8, c=4, d=2, f=64), cabi.FP32, 0, ["simt (", "one output per thread"]),
    # output contiguous along the right operand: the planner swaps the roles
    ("bi,io->bo", dict(b=8192, i=4096, o=4096), cabi.BF16, 0, ["tc kind=bf16", "A=MN B=K", "operands swapped"]),
    ("zabcd,zcdef->zabef", dict(z=64, a=48, b=48, c=48, d=48, e=48, f=48), cabi.FP64, 0,
     ["tc kind=fp64-dmma", "A=MN B=K", "operands swapped", "64 slab(s), counted by the kernel"]),
]


@pytest.mark.parametrize("expr,sizes,dt,comp,frags", PLAN_CASES)
def test_lowering_decisions(expr, sizes, dt, comp, frags, monkeypatch):
    monkeypatch.delenv("EIR_TC_MIN_OPS", raising=False)
    monkeypatch.delenv("EIR_TC_MIN_UTIL", raising=False)
    il, ir, io, names = binary.parse_binary(expr)
    sz = {i: sizes[c] for i, c in enumerate(names)}
    dto = cabi.FP64 if dt == cabi.FP64 else cabi.FP32
    plan = cabi.ContractPlan(binary.contraction_dims(il, ir, io, sz), dt, dt, dto, comp)
    d = plan.describe()
    for f in frags:
        assert f in d, d


@pytest.mark.parametrize("expr,sizes,direct", [
    ("mk,nk->nm", dict(m=32, n=32, k=64), True),        # K <= 64
    ("mk,nk->nm", dict(m=32, n=32, k=65), False),       # K > 64 and outputs x K > 2^16
    ("mk,nk->nm", dict(m=2, n=2, k=16384), True),       # outputs x K = 2^16
    ("mk,nk->nm", dict(m=2, n=2, k=16385), False),
    ("mn,n->mn", dict(m=2048, n=2047), True),           # no K dim, 2^22 - 2048 outputs
    ("mn,n->mn", dict(m=2048, n=2048), False),          # 2^22 outputs
])
def test_simt_direct_eligibility(expr, sizes, direct, monkeypatch):
    # the one-output-per-thread CUDA-core kernel takes fewer than 2^22 outputs
    # with K <= 64 or outputs x K <= 2^16; EIR_SIMT_DIRECT=0 keeps the tiled one
    il, ir, io, names = binary.parse_binary(expr)
    sz = {i: sizes[c] for i, c in enumerate(names)}
    dims = binary.contraction_dims(il, ir, io, sz)
    monkeypatch.delenv("EIR_SIMT_DIRECT", raising=False)
    plan = cabi.ContractPlan(dims, cabi.FP32, cabi.FP32, cabi.FP32, flags=cabi.FLAG_FORCE_SIMT)
    assert ("one output per thread" in plan.describe()) == direct, plan.describe()
    monkeypatch.setenv("EIR_SIMT_DIRECT", "0")
    plan = cabi.ContractPlan(dims, cabi.FP32, cabi.FP32, cabi.FP32, flags=cabi.FLAG_FORCE_SIMT)
    assert "one output per thread" not in plan.describe(), plan.describe()


def test_error_codes():
    dims = [(cabi.DIM_M, 4, 1, 0, 1, 0), (cabi.DIM_N, 4, 0, 1, 4, 0), (cabi.DIM_K, 4, 4, 4, 0, 0)]
    with pytest.raises(cabi.EirError) as e:
        cabi.ContractPlan(dims, cabi.FP64, cabi.FP32, cabi.FP32)
    assert e.value.code == 9  # INVALID_DTYPE
    with pytest.raises(cabi.EirError) as e:
        cabi.ContractPlan(dims, cabi.FP32, cabi.FP32, cabi.FP32, first=cabi.KTYPE_RELU)
    assert e.value.code == 10  # INVALID_KTYPE
    with pytest.raises(cabi.EirError) as e:
        cabi.ContractPlan([(7, 4, 1, 1, 1, 0)], cabi.FP32, cabi.FP32, cabi.FP32)
    assert e.value.code == 52
    assert cabi.lib().eir_contract(None, None, None, None, None, None) == 52
    plan = cabi.ContractPlan(dims, cabi.FP32, cabi.FP32, cabi.FP32)
    assert plan.num_ops == 2 * 4 * 4 * 4 - 4 * 4  # ZERO first touch (BinaryContraction.cpp:459-462)


def test_direct_kernel_division_by_multiplication():
    """the direct CUDA-core kernel splits an index x < 2^32 by a dim size d
    as q = (x * M) >> 64 with M = UINT64_MAX // d + 1 = ceil(2^64 / d) (the
    planner's magic_of); exact for every such x and 2 <= d < 2^32 (Lemire,
    Kaser, Kurz 2019). Checked on the edges of every multiple it can miss"""
    rng = random.Random(7)
    divisors = list(range(2, 300)) + [2 ** k for k in range(1, 32)] + [2 ** k - 1 for k in range(2, 33)] + \
        [rng.randrange(2, 2 ** 32) for _ in range(300)]
    for d in divisors:
        m = (2 ** 64 - 1) // d + 1
        qs = {0, 1, 2, (2 ** 32 - 1) // d} | {rng.randrange(0, (2 ** 32 - 1) // d + 1) for _ in range(20)}
        for q in qs:
            for x in (q * d - 1, q * d, q * d + d - 1):
                if 0 <= x < 2 ** 32:
                    assert (x * m) >> 64 == x // d, (x, d)
