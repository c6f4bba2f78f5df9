"""Batch-sharded config 5 on two GPUs through torchrun (einsum_ir_b200.sharded):
the copy-engine gather of finished z-slabs (eir_contract_gather, FP64 and
TF32), the fused gather (every rank's epilogue stores into all ranks' outputs
over NVLink) and the NCCL all-gather path, each checked on one z-slab of every
rank's block against torch. Skipped with fewer than 2 GPUs."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu


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
