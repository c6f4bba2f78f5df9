"""Batch-sharded config 5 on two GPUs through torchrun (einsum_ir_b200.sharded):
the copy-engine gather of finished z-slabs (eir_contract_gather, FP64 and
TF32), the fused gather (every rank's epilogue stores into all ranks' outputs
over NVLink) and the NCCL all-gather path, each checked on one z-slab of every
rank's block against torch. Skipped with fewer than 2 GPUs. The C++ entry
point (ShardedContraction, through the bench_sharded driver and its
file-based handle exchange) runs with one rank on any GPU and with two ranks
on two GPUs; the driver checks the first slab of every rank's block in its
gathered output against the FP64 CUDA-core contraction of that slab."""
from __future__ import annotations

import json
import os
import subprocess
import sys

from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
PKG = Path(__file__).resolve().parents[1] / "einsum_ir_b200"


def _gpus() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("args,tol", [([], 1e-12), (["--fp32", "--tf32"], 3e-3), (["--fused"], 1e-12), (["--nccl"], 1e-12)])
def test_sharded_two_ranks(args, tol):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "20", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29533",
           "-m", "einsum_ir_b200.sharded"] + args
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("{")][-1]
    res = json.loads(line)
    assert res["gpus"] == 2 and res["rel_err_check"] <= tol, res
    assert ("NCCL" in res["gather"]) == ("--nccl" in args), res
    if not args or args == ["--fp32", "--tf32"]:
        assert "copy engines" in res["gather"], res


def _bench_sharded(tmp_path, world, z, n, dtype):
    procs = [subprocess.Popen([str(PKG / "bench_sharded"), str(r), str(world), str(tmp_path), str(z), str(n),
                               dtype], stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
             for r in range(world)]
    outs = []
    for p in procs:
        out, err = p.communicate(timeout=300)
        outs.append((p.returncode, out, err))
    for rc, out, err in outs:
        assert rc == 0, out[-2000:] + err[-2000:]
        assert "CSV_DATA: einsum_ir_b200,bench_sharded," in out
    return outs


@pytest.mark.parametrize("dtype", ["FP64", "FP32"])
def test_cpp_sharded_contraction_one_rank(cuda, tmp_path, dtype):
    _bench_sharded(tmp_path, 1, 8, 16, dtype)


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_cpp_sharded_contraction_two_ranks(tmp_path):
    _bench_sharded(tmp_path, 2, 8, 24, "FP64")
