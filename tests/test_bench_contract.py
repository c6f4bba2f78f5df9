"""CPU tests of bench.py's reference arm: the JSON line the benchmark driver
reads (one process, and under torchrun where only rank 0 may print). The
arm times the reference's own scalar contraction backend (oracle/_ref) on a
bounded sample of the config 5 workload, on the host cores; skipped when that
library was not built."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

from tests import _refscalar

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.skipif(not _refscalar.available(),
                                reason="reference scalar library not built (needs the reference sources)")


def _lines(stdout: str):
    return [json.loads(l) for l in stdout.splitlines() if l.startswith("{")]


def _check(line, gpus):
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["n_gpus"] == gpus
    assert line["metric"] == "Einsum-tree TFLOP/s" and line["unit"] == "TFLOP/s" and line["higher_is_better"]
    assert line["value"] > 0 and line["warmup"] >= 3 and line["steps"] == 1
    assert "zabcd,zcdef->zabef" in line["config"]["workload"]
    cb = line["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == line["value"] and cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_one_process():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1, r.stdout
    _check(lines[0], 1)


def test_reference_arm_under_torchrun_prints_once():
    cmd = ["timeout", "-k", "20", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29611",
           str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=700, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1, r.stdout  # rank 0 only; rank 1 exits without work
    _check(lines[0], 2)
