"""Sample suites through the drivers on the GPU (einsum_ir_b200.run_samples,
the counterpart of the reference's samples/tools/bench_einsum_ir.sh).

* The committed synthetic suite (tests/golden/samples/, written by
  tests/golden/make_samples.py: seeded random tensor networks in the suites'
  expression and tree line formats) always runs, in expression mode (1) and
  tree mode (2): every setting must finish, pass its driver's own check, and
  its result (dumped with EIR_DRIVER_DUMP) must match the CPU oracle evaluated
  on the same input values with FP32 intermediates (1e-5).
* With EIR_SAMPLES_DIR set to a directory laid out as the reference's
  samples/, its suite files run too (they are the caller's data, not part of
  the repository): every setting must finish and match its FP64 CUDA-core
  solution within the north_star tolerance (FP32 1e-4); the drivers' own exit
  status uses the reference driver's stricter 1e-5 bound, which a deep FP32
  tree may exceed through FP32 intermediates alone.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

import pytest

from einsum_ir_b200 import run_samples as rs
from tests import _oracle, _tree

pytestmark = pytest.mark.gpu
SAMPLES = os.environ.get("EIR_SAMPLES_DIR")
SYNTHETIC = Path(__file__).resolve().parent / "golden" / "samples"
TABLES = {1: {"synthetic": "synthetic.cfg"}, 2: {"synthetic": "synthetic_et.cfg"}}


@pytest.mark.parametrize("mode", [1, 2])
def test_synthetic_suite_runner_and_oracle(cuda, tmp_path, mode, monkeypatch):
    monkeypatch.setenv("EIR_DRIVER_TIME_MS", "20")
    rows = rs.run(SYNTHETIC, ["synthetic"], mode, 1, "FP32", tmp_path / "logs", table=TABLES[mode])
    assert len(rows) == 8
    bad = [r for r in rows if r["status"] != "ok" or "rel_err" not in r]
    assert not bad, bad
    # every setting once more with its inputs and result dumped, against the oracle
    for line, args in rs.parse_setting_file(SYNTHETIC / TABLES[mode]["synthetic"]):
        d = tmp_path / f"dump{line}"
        d.mkdir()
        env = dict(os.environ, EIR_DRIVER_DUMP=str(d))
        r = subprocess.run(rs.driver_command(mode, args, "FP32"), capture_output=True, text=True, env=env,
                           timeout=300)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
        man, tensor = _tree.load_dump(d)
        got = tensor("out")[2]
        if mode == 1:
            n_in = len([k for k in man if k.startswith("in")])
            ref = _tree.eval_tree(man["expr"], man["sizes"], man["path"],
                                  [tensor(f"in{t}")[2] for t in range(n_in)], model="fp32")
        else:
            nodes, leaves, sz = [], {}, {}
            for i in range(len([k for k in man if k.startswith("node")])):
                f = man[f"node{i}"].split()
                ids = [] if f[1] == "-" else [int(x) for x in f[1].split(",")]
                ch = [] if f[3] == "-" else [int(x) for x in f[3].split(",")]
                nodes.append((ids, ch))
                if not ch:
                    lids, lsz, leaves[i] = tensor(f"leaf{i}")
                    sz.update(zip(lids, lsz))
            oids, osz, _ = tensor("out")
            sz.update(zip(oids, osz))
            ref = _tree.eval_nodes(nodes, sz, leaves, "fp32")
        assert _oracle.rel_err(got, ref) <= 1e-5, f"line {line}: {args}"


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
