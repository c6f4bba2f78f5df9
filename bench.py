"""Benchmark of the einsum_ir B200 hot path (driver contract: one JSON line).

Workload: the strided binary contraction
``akmj,njk->anm`` with a=16, k=32, m=512, j=64, n=512 (M = a*m = 8192,
N = 512, K = k*j = 2048), BF16 inputs drawn U[-1,1] from a seed, FP32
accumulation and output. A step is one contraction through the C-ABI
(``eir_contract``: pre-permute of the right operand + tcgen05 kernel).

* ``value``: TFLOP/s with inputs resident in HBM; L2 is flushed (256 MiB
  write) before every step, outside the per-step CUDA-event window, so each
  step reads its operands from HBM.
* ``e2e``: the same step through the same public call with host buffers:
  pinned host -> device copies of both operands, the contraction and the
  device -> host copy of the result inside the timed window.
* ``roofline``: the tensor-core kernel alone, timed live by the library's
  per-plan event timing (eir_plan_profile), against the measured dense BF16
  peak; ``traffic`` is the DRAM bytes per launch from the committed ncu
  capture of that kernel.
* ``cpu_baseline``: the CPU oracle (a C restatement of the reference loop
  engine; the reference's libxsmm build is not available) on one ``a`` slab.

Multi-GPU (torchrun, one process per GPU): every rank contracts its own
a-slab of a job with a = 16 * world_size (weak scaling, no data-path
collective); ``value`` = all ranks' FLOPs / max-over-ranks time.
``--impl reference`` times the CPU oracle port on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SIZES = dict(a=16, k=32, m=512, j=64, n=512)
EXPR = "akmj,njk->anm"
WORKLOAD = "binary contraction akmj,njk->anm (a=16,k=32,m=512,j=64,n=512; BF16 in, FP32 acc/out)"
METRIC = "Einsum-tree TFLOP/s"
FLUSH_BYTES = 256 * 1024 * 1024


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    return 1590.0, 6650.0, "fallback"


def _profile_traffic():
    """DRAM bytes per launch of the tensor-core kernel from the committed ncu summary."""
    f = ROOT / "profiles" / "tc_pair_contract_bf16_cfg2.txt"
    if not f.exists():
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", f.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self, idle_mhz: float = 600.0):
        rows = []
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        load = [r for r in rows if r[0] > idle_mhz] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in load for i, v in enumerate(r[2]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in load), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def _cpu_oracle_sample(threads: int, budget_s: float = 12.0):
    """Time the CPU oracle on a-slabs of the workload (the oracle is test
    infrastructure; here it only provides the reported CPU baseline)."""
    import numpy as np
    from tests import _oracle
    from einsum_ir_b200 import binary, cabi
    s = dict(SIZES, a=1)
    il, ir, io, names = binary.parse_binary(EXPR)
    sz = {i: s[c] for i, c in enumerate(names)}
    dims = binary.contraction_dims(il, ir, io, sz)
    rng = np.random.default_rng(0)
    def bf16(n):
        x = (rng.random(n, dtype=np.float32) * 2 - 1).view(np.uint32)
        return ((x + 0x7FFF + ((x >> 16) & 1)) >> 16).astype(np.uint16)
    nl = int(np.prod([sz[i] for i in il]))
    nr = int(np.prod([sz[i] for i in ir]))
    no = int(np.prod([sz[i] for i in io]))
    l, r, o = bf16(nl), bf16(nr), np.zeros(no, dtype=np.float32)
    flops = 2.0 * nl * s["n"]  # 2*M*N*K for one a slab
    slabs, t0 = 0, time.perf_counter()
    while True:
        _oracle.contract(dims, l, r, o, None, cabi.BF16, cabi.BF16, cabi.FP32, 0,
                         cabi.KTYPE_ZERO, cabi.KTYPE_UNDEFINED, threads)
        slabs += 1
        el = time.perf_counter() - t0
        if el > budget_s or slabs >= 16:
            break
    return {"value": flops * slabs / el / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{slabs} a-slab(s) of the workload (a=1: M=512,N=512,K=2048), "
                      f"{el:.1f} s, CPU oracle restating the reference loop engine "
                      "(reference libxsmm TPP build unavailable: libxsmm absent)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    # each step = one a-slab (1/16 of the workload) on all host threads
    for _ in range(args.warmup):
        _cpu_oracle_sample(threads, budget_s=0.0)
    vals = [_cpu_oracle_sample(threads, budget_s=0.0) for _ in range(args.steps)]
    cb = vals[-1]
    val = statistics.median(v["value"] for v in vals)
    times = [2.0 * SIZES["m"] * SIZES["n"] * SIZES["k"] * SIZES["j"] / (v["value"] * 1e12) for v in vals]
    cb = dict(cb, value=val, sample=f"{args.steps} steps of one a-slab each (a=1: M=512,N=512,K=2048) "
              "through the CPU oracle restating the reference loop engine (reference libxsmm TPP "
              "build unavailable: libxsmm absent); value = median slab throughput")
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * statistics.mean(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD + " [sampled: a-slabs]"},
            "cpu_baseline": cb,
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist
    from einsum_ir_b200 import binary, cabi

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    il, ir, io, names = binary.parse_binary(EXPR)
    sz = {i: SIZES[c] for i, c in enumerate(names)}
    dims = binary.contraction_dims(il, ir, io, sz)
    plan = cabi.ContractPlan(dims, cabi.BF16, cabi.BF16, cabi.FP32)
    flops_alg = 2.0 * SIZES["a"] * SIZES["m"] * SIZES["n"] * SIZES["k"] * SIZES["j"]

    g = torch.Generator().manual_seed(1234 + rank)
    shp = lambda ids: [sz[i] for i in ids]
    l_h = (torch.rand(shp(il), generator=g) * 2 - 1).to(torch.bfloat16).pin_memory()
    r_h = (torch.rand(shp(ir), generator=g) * 2 - 1).to(torch.bfloat16).pin_memory()
    o_h = torch.empty(shp(io), dtype=torch.float32).pin_memory()
    l = l_h.to(dev)
    r = r_h.to(dev)
    o = torch.empty(shp(io), dtype=torch.float32, device=dev)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def reduce_max(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timing: CUDA events around each step only (per-launch
    # events inside a step would separate the pre-permute from the contraction
    # kernel and cost the programmatic-dependent-launch overlap)
    for _ in range(args.warmup):
        plan.contract(l, r, o, stream=sp)
    barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    launches0 = cabi.launch_count()
    barrier()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            ev[i][0].record(stream)
            plan.contract(l, r, o, stream=sp)
            ev[i][1].record(stream)
        barrier()
    launches = cabi.launch_count() - launches0
    step_ms = sum(a.elapsed_time(b) for a, b in ev)
    step_ms_max = reduce_max(step_ms)

    # ---- the same K steps again with CUDA events around the contraction
    # kernel's own launch (library timing on the launch stream) for the roofline
    plan.profile(True)
    plan.profile_read()
    for i in range(args.steps):
        flush.fill_(i & 0xFF)
        plan.contract(l, r, o, stream=sp)
    barrier()
    kern_ms, kern_n = plan.profile_read()
    plan.profile(False)
    kern_ms_avg = reduce_max(kern_ms / max(1, kern_n))
    value = world * flops_alg * args.steps / (step_ms_max * 1e-3) / 1e12

    # ---- end-to-end through the same public call with host buffers
    for _ in range(min(args.warmup, 3)):
        l.copy_(l_h, non_blocking=True)
        r.copy_(r_h, non_blocking=True)
        plan.contract(l, r, o, stream=sp)
        o_h.copy_(o, non_blocking=True)
    barrier()
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    for i in range(args.steps):
        flush.fill_(i & 0xFF)
        e2e_ev[i][0].record(stream)
        l.copy_(l_h, non_blocking=True)
        r.copy_(r_h, non_blocking=True)
        plan.contract(l, r, o, stream=sp)
        o_h.copy_(o, non_blocking=True)
        e2e_ev[i][1].record(stream)
    barrier()
    e2e_ms = reduce_max(sum(a.elapsed_time(b) for a, b in e2e_ev))
    e2e_value = world * flops_alg * args.steps / (e2e_ms * 1e-3) / 1e12

    # correctness spot check of the last result against a torch fp32 einsum
    ref = torch.einsum(EXPR, l.float(), r.float())
    rel = float((o - ref).norm() / ref.norm())
    cabi.check_device_errors(sp)

    peak_tf, hbm, peak_src = _peaks()
    kernel_name = ("tc_pair_contract_kernel<bf16,256,KSUB>" if "pair" in plan.describe()
                   else "tc_contract_kernel<bf16,BN,KSUB>")
    achieved = flops_alg / (kern_ms_avg * 1e-3) / 1e12
    traffic = _profile_traffic()
    line = None
    if rank == 0:
        cpu = _cpu_oracle_sample(os.cpu_count() or 1) if world == 1 else None
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "per_rank": "a=16 slab of a=16*world_size",
                       "l2": "flushed before every step (256 MiB write, outside the step window)",
                       "plan": plan.describe(), "rel_err_vs_torch_fp32": rel},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": l.numel() * 2 + r.numel() * 2,
                    "d2h_bytes_per_step": o.numel() * 4},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf,
                         "unit": "TFLOP/s", "frac": achieved / peak_tf, "traffic": traffic,
                         "kernel": kernel_name, "peak_source": peak_src,
                         "kernel_ms": kern_ms_avg,
                         "kernel_timing": "events around the kernel launch, second pass of the K steps"},
            "cpu_baseline": cpu,
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
