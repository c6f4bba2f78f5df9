"""Runs sample suites of einsum settings through this backend's drivers: the
counterpart of the reference's samples/tools/bench_einsum_ir.sh.

    python -m einsum_ir_b200.run_samples --samples DIR [-k keys] [-d mode]
        [-r reps] [--dtype FP32] [-l log_dir] [--csv summary.csv] [--dry-run]

DIR is a samples directory laid out as the reference's ``samples/`` (the
suites are data files of the caller, not part of this package). Each line of
a setting file holds the driver arguments of one setting:
``"expression" "sizes" "path"`` (modes 0 and 1: run by ``bench_expression``
with ``<dtype> 0 1`` as the reference script does) or ``"tree" "sizes"``
(mode 2: ``bench_tree <dtype>``). Every driver run checks its result against
an FP64 CUDA-core solution of the same inputs and exits non-zero when the
error is large; a setting counts as failed then. The GPU backend has a single
layout policy for intermediates, so modes 0 and 1 run the same way.

Output: one log per key (driver output, as the reference script writes) and
a summary line per setting (key, line, status, flops, eval seconds, GFLOPS,
relative error against the FP64 solution). A driver fails a setting above
the reference driver's bound (FP32 1e-5, FP64 1e-12; src/bench_expression.cpp
:535-541), which here is checked against FP64 rather than an FP32 library
result.
"""
from __future__ import annotations

import argparse
import csv
import io
import os
import re
import shlex
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent

# key -> setting file, as samples/tools/bench_einsum_ir.sh:95-118
EXPRESSION_SETTINGS = {
    "syn": "einsum_benchmark/synthetic.cfg",
    "tt": "tensor_decomp/tt.cfg",
    "fctn": "tensor_decomp/fctn.cfg",
    "tw": "tensor_decomp/tw.cfg",
    "getd": "tensor_decomp/getd.cfg",
    "trn": "tensor_layers/trn.cfg",
    "mera": "einsum_benchmark/str_nw_mera_open_26.cfg",
    "tnlm": "einsum_benchmark/lm_first_last_brackets_4_16d.cfg",
    "tccg_blocked_reordered": "tccg/settings_blocked_reordered.cfg",
    "tccg_blocked": "tccg/settings_blocked.cfg",
    "fc": "tensor_layers/fc.cfg",
}
TREE_SETTINGS = {
    "syn": "einsum_benchmark/synthetic_et.cfg",
    "tt": "tensor_decomp/tt_et.cfg",
    "fctn": "tensor_decomp/fctn_et.cfg",
    "tw": "tensor_decomp/tw_et.cfg",
    "getd": "tensor_decomp/getd_et.cfg",
    "trn": "tensor_layers/trn_et.cfg",
    "mera": "einsum_benchmark/str_nw_mera_open_26_et.cfg",
    "tnlm": "einsum_benchmark/lm_first_last_brackets_4_16d_et.cfg",
}
# further TCCG setting files (expression form) this runner also accepts
EXTRA_EXPRESSION_SETTINGS = {
    "tccg_default": "tccg/settings_default.cfg",
    "tccg_adjusted": "tccg/settings_adjusted.cfg",
    "tccg_batch": "tccg/settings_batch.cfg",
    "tccg_full": "tccg/settings_full.cfg",
}


def settings_for(mode: int) -> dict:
    if mode == 2:
        return dict(TREE_SETTINGS)
    return {**EXPRESSION_SETTINGS, **EXTRA_EXPRESSION_SETTINGS}


def parse_setting_file(path: Path) -> list:
    """(line number, argument list) of every non-empty line"""
    out = []
    for i, line in enumerate(path.read_text().splitlines(), 1):
        if line.strip():
            out.append((i, shlex.split(line)))
    return out


_CSV = re.compile(r"^CSV_DATA: (.*)$", re.M)
_REL = re.compile(r"^\s*relative error:\s*(\S+)\s*$", re.M)


def parse_driver_output(text: str) -> dict:
    """flops / eval time / GFLOPS from the driver's CSV_DATA line, and the
    relative error of its FP64 check"""
    m = _CSV.search(text)
    if not m:
        return {}
    e = _REL.search(text)
    rel = {"rel_err": float(e.group(1))} if e else {}
    row = next(csv.reader(io.StringIO(m.group(1))))
    # bench_expression: backend,expr,sizes,path,flops,t_compile,t_eval,gf_eval,gf_total
    # bench_tree:       backend,tree,sizes,flops,t_compile,t_eval,gf_eval,gf_total
    nums = row[-5:]
    try:
        return dict(flops=int(float(nums[0])), t_compile=float(nums[1]), t_eval=float(nums[2]),
                    gflops=float(nums[3]), **rel)
    except ValueError:
        return {}


def driver_command(mode: int, args: list, dtype: str) -> list:
    if mode == 2:
        return [str(PKG / "bench_tree")] + args + [dtype]
    return [str(PKG / "bench_expression")] + args + [dtype, "0", "1"]


def run(samples: Path, keys: list, mode: int, reps: int, dtype: str, log_dir: Path,
        dry_run: bool = False, timeout: float = 600.0, max_per_key: int = 0, table: dict | None = None) -> list:
    """runs the settings of `keys`; `table` maps keys to setting files under
    `samples` (default: the reference's suite layout, settings_for(mode))"""
    table = settings_for(mode) if table is None else table
    rows = []
    for key in keys:
        if key not in table:
            raise SystemExit(f"invalid benchmark key '{key}' (available: {', '.join(sorted(table))})")
        f = samples / table[key]
        if not f.exists():
            raise SystemExit(f"setting file {f} not found")
        log = log_dir / key / (f"einsum_ir_b200_mode_{mode}.log")
        if not dry_run:
            log.parent.mkdir(parents=True, exist_ok=True)
            log.write_text("")
        settings = parse_setting_file(f)
        if max_per_key > 0 and len(settings) > max_per_key:
            # an even spread over the file
            step = len(settings) / max_per_key
            settings = [settings[int(i * step)] for i in range(max_per_key)]
        for line, args in settings:
            cmd = driver_command(mode, args, dtype)
            if dry_run:
                rows.append(dict(key=key, line=line, cmd=cmd))
                continue
            for _ in range(reps):
                try:
                    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
                    text, rc = r.stdout + r.stderr, r.returncode
                except subprocess.TimeoutExpired:
                    text, rc = "timeout\n", -1
                with open(log, "a") as fh:
                    fh.write(text)
                res = parse_driver_output(text)
                rows.append(dict(key=key, line=line, status="ok" if rc == 0 else f"failed({rc})", **res))
    return rows


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--samples", required=True, type=Path, help="samples directory (reference layout)")
    ap.add_argument("-k", "--keys", default="all", help="comma-separated keys or 'all'")
    ap.add_argument("-d", "--mode", type=int, default=1, choices=(0, 1, 2))
    ap.add_argument("-r", "--reps", type=int, default=1)
    ap.add_argument("--dtype", default="FP32")
    ap.add_argument("-l", "--log-dir", type=Path, default=Path("logs"))
    ap.add_argument("--csv", type=Path, default=None, help="write the summary here")
    ap.add_argument("--dry-run", action="store_true", help="print the driver commands only")
    ap.add_argument("--max-per-key", type=int, default=0,
                    help="run at most this many settings per key (evenly spread; 0 = all)")
    ap.add_argument("--time-ms", type=float, default=None,
                    help="timing budget per setting for the drivers (EIR_DRIVER_TIME_MS; default 500)")
    a = ap.parse_args(argv)
    table = settings_for(a.mode)
    keys = sorted(table) if a.keys == "all" else [k for k in a.keys.split(",") if k]
    if a.keys == "all":
        keys = [k for k in keys if (a.samples / table[k]).exists()]
    if a.time_ms is not None:
        os.environ["EIR_DRIVER_TIME_MS"] = str(a.time_ms)
    rows = run(a.samples, keys, a.mode, a.reps, a.dtype, a.log_dir, a.dry_run, max_per_key=a.max_per_key)
    if a.dry_run:
        for r in rows:
            print(r["key"], r["line"], " ".join(shlex.quote(c) for c in r["cmd"]))
        return 0
    fields = ["key", "line", "status", "flops", "t_eval", "gflops", "rel_err"]
    out = open(a.csv, "w", newline="") if a.csv else sys.stdout
    w = csv.DictWriter(out, fieldnames=fields, extrasaction="ignore")
    w.writeheader()
    for r in rows:
        w.writerow(r)
    if a.csv:
        out.close()
    failed = [r for r in rows if r["status"] != "ok"]
    print(f"{len(rows) - len(failed)} of {len(rows)} settings ok", file=sys.stderr)
    return 1 if failed else 0


if __name__ == "__main__":
    sys.exit(main())
