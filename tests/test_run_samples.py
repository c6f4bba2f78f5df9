"""The sample-suite runner (einsum_ir_b200.run_samples, the counterpart of the
reference's samples/tools/bench_einsum_ir.sh) on made-up setting files: key
table, line parsing, driver command lines, per-key caps and the parsing of a
driver report. No GPU."""
from __future__ import annotations

from pathlib import Path

from einsum_ir_b200 import run_samples as rs


def _samples(tmp_path: Path) -> Path:
    (tmp_path / "tccg").mkdir()
    (tmp_path / "tccg" / "settings_default.cfg").write_text(
        '"ab,bc->ac" "4,5,6" "(0,1)"\n\n"abc,cd->abd" "2,3,4,5" "(0,1)"\n"xy,yz->xz" "7,8,9" "(0,1)"\n')
    (tmp_path / "einsum_benchmark").mkdir()
    (tmp_path / "einsum_benchmark" / "synthetic_et.cfg").write_text('"[0,1],[1,2]->[0,2]" "3,4,5"\n')
    return tmp_path


def test_setting_files_and_commands(tmp_path):
    s = _samples(tmp_path)
    lines = rs.parse_setting_file(s / "tccg" / "settings_default.cfg")
    assert [n for n, _ in lines] == [1, 3, 4]
    assert lines[0][1] == ["ab,bc->ac", "4,5,6", "(0,1)"]
    rows = rs.run(s, ["tccg_default"], 1, 1, "FP32", tmp_path / "logs", dry_run=True)
    assert len(rows) == 3
    assert rows[0]["cmd"][0].endswith("bench_expression") and rows[0]["cmd"][-3:] == ["FP32", "0", "1"]
    rows = rs.run(s, ["tccg_default"], 1, 1, "FP32", tmp_path / "logs", dry_run=True, max_per_key=2)
    assert [r["line"] for r in rows] == [1, 3]
    rows = rs.run(s, ["syn"], 2, 1, "FP64", tmp_path / "logs", dry_run=True)
    assert rows[0]["cmd"][0].endswith("bench_tree") and rows[0]["cmd"][1:] == ["[0,1],[1,2]->[0,2]", "3,4,5", "FP64"]
    # the reference script's key tables
    assert set(rs.TREE_SETTINGS) < set(rs.EXPRESSION_SETTINGS)
    assert rs.settings_for(2) == rs.TREE_SETTINGS


def test_driver_report_parsing():
    text = ("  #flops:         1000\n"
            'CSV_DATA: einsum_ir_b200,"ab,bc->ac","4,5,6","(0,1)",1000,0.5,0.001,1,0.002\n'
            "*** comparing solution ***:\n  relative error:                               3.5e-07\n")
    r = rs.parse_driver_output(text)
    assert r == dict(flops=1000, t_compile=0.5, t_eval=0.001, gflops=1.0, rel_err=3.5e-07)
    tree = 'CSV_DATA: einsum_ir_b200,"[0,1],[1,2]->[0,2]","3,4,5",60,0.1,2e-06,0.03,0.0006\n'
    assert rs.parse_driver_output(tree)["flops"] == 60
    assert rs.parse_driver_output("no report") == {}
