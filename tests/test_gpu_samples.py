"""Sample suites through the drivers on the GPU (einsum_ir_b200.run_samples).

The suites are the caller's data files: set EIR_SAMPLES_DIR to a directory
laid out as the reference's samples/ to run this test; without it the test
is skipped. Every setting must finish and match its FP64 CUDA-core solution
within the north_star tolerance (FP32 1e-4); the drivers' own exit status
uses the reference driver's stricter 1e-5 bound, which a deep FP32 tree may
exceed through FP32 intermediates alone.
"""
from __future__ import annotations

import os
from pathlib import Path

import pytest

from einsum_ir_b200 import run_samples as rs

pytestmark = pytest.mark.gpu
SAMPLES = os.environ.get("EIR_SAMPLES_DIR")


@pytest.mark.skipif(not SAMPLES, reason="EIR_SAMPLES_DIR not set (suite files are not part of the repository)")
@pytest.mark.parametrize("mode", [1, 2])
def test_sample_suites(cuda, tmp_path, mode):
    os.environ["EIR_DRIVER_TIME_MS"] = "20"
    table = rs.settings_for(mode)
    keys = sorted(k for k in table if (Path(SAMPLES) / table[k]).exists())
    assert keys
    rows = rs.run(Path(SAMPLES), keys, mode, 1, "FP32", tmp_path, max_per_key=2)
    bad = [r for r in rows if "rel_err" not in r or r["rel_err"] > 1e-4]
    assert not bad, bad
