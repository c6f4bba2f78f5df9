"""Benchmark of the einsum_ir B200 hot path (driver contract: one JSON line).

Workload (the largest config that fits one GPU and the
one the 8-GPU target is quoted on): the batch-sharded high-order contraction
``zabcd,zcdef->zabef`` with z=64, a=b=c=d=e=f=48, FP64 on the FP64 tensor
cores (C = z 64, M = ab 2304, N = ef 2304, K = cd 2304: 2 x 64 x 2304^3 =
1.566e12 flop per step), inputs U[-1,1] from a seed. Each operand is 2.72 GB,
far larger than L2 (126 MB), so every step reads them from HBM (no flush).

* N = 1: a step is one ``eir_contract`` of the whole job (one DMMA launch).
* N > 1 (torchrun, one process per GPU): z is split into N contiguous blocks;
  rank r contracts its block and ``eir_contract_gather`` copies every finished
  z-slab into the other ranks' full outputs (copy engines over NVLink, CUDA IPC
  mappings) while the kernel computes the next slabs, so a step ends with the
  full output on every GPU. Total work is fixed: ``"scaling": "strong"``.
* ``value``: TFLOP/s of the whole job, CUDA events around each step on the
  launching stream, max over ranks.
* ``e2e``: the same job through the same public calls with HOST buffers: per
  step the pinned-host -> device copy of this rank's input blocks, the
  contraction (and gather), and the device -> host copy of this rank's block of
  the result, pipelined over groups of z-slabs (copies of one group overlap the
  kernel of the previous one).
* ``roofline``: the contraction kernel alone (library event timing around the
  kernel launch, a second pass of the K steps) against the FP64 peak measured
  in this run: cuBLAS DGEMM (torch.matmul, 8192^3 FP64) best of 5, because
  MEASURED_PEAKS.json carries no FP64 figure.
* ``cpu_baseline`` (rank 0, N = 1): the reference's own scalar contraction
  backend (BinaryContractionScalar compiled from the reference sources into
  oracle/_ref; its libxsmm backend cannot be built: libxsmm is absent) on a
  bounded sample of the workload, with torch's CPU einsum (a BLAS DGEMM) as a
  labelled second stand-in.
``--impl reference`` times that same reference scalar backend on the same
sample, every step, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
# eir_contract_gather keeps one copy stream per peer waiting on the kernel's
# slab counters; with CUDA's default 8 hardware work queues those streams
# share queues with the compute stream and with one another, and a blocked
# wait then holds back the work queued behind it. Must be set before the CUDA
# context exists.
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

EXPR = "zabcd,zcdef->zabef"
SIZES = dict(z=64, a=48, b=48, c=48, d=48, e=48, f=48)
WORKLOAD = ("batch-sharded contraction zabcd,zcdef->zabef (z=64, a=b=c=d=e=f=48; FP64; "
            "C=z 64, M=ab 2304, N=ef 2304, K=cd 2304)")
METRIC = "Einsum-tree TFLOP/s"
FLOPS = 2.0 * 64 * 2304 ** 3
# bounded CPU sample of the workload: z=1, a=1, b=16 (2 x 16 x 2304 x 2304 flop)
SAMPLE = dict(z=1, a=1, b=16, c=48, d=48, e=48, f=48)


def _lscpu():
    model, cores = platform.processor() or "unknown", os.cpu_count() or 1
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for l in out.splitlines():
            if l.startswith("Model name:"):
                model = l.split(":", 1)[1].strip()
    except (OSError, subprocess.SubprocessError):
        pass
    return model, cores


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
                rows.append((float(f[1]), float(f[2]), float(f[3]), f[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        load = [r for r in rows if r[0] > idle_mhz] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in load for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in load), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------ CPU baselines
def _ref_sample():
    """(reference scalar contraction of the sample, inputs, output, flops)"""
    import numpy as np
    from tests import _refscalar
    from einsum_ir_b200 import binary
    il, ir, io, names = binary.parse_binary(EXPR)
    sz = {i: SAMPLE[c] for i, c in enumerate(names)}
    rng = np.random.default_rng(0)
    l = rng.uniform(-1, 1, [sz[i] for i in il])
    r = rng.uniform(-1, 1, [sz[i] for i in ir])
    o = np.zeros([sz[i] for i in io])
    c = _refscalar.Contraction(il, ir, io, sz, dtype=1, first=0, threads=os.cpu_count() or 1)
    return c, l, r, o


def _ref_available() -> bool:
    from tests import _refscalar
    return _refscalar.available()


REF_DESC = ("reference scalar contraction backend (backend::BinaryContractionScalar, compiled from "
            "the reference sources into oracle/_ref; the reference's libxsmm TPP backend is "
            "unbuildable here: libxsmm absent)")
SAMPLE_DESC = "z=1, a=1, b=16 block of the workload (M=16, N=2304, K=2304: 1.70e8 flop)"


def _time_ref_step(c, l, r, o) -> float:
    t0 = time.perf_counter()
    c.contract(l, r, o)
    return time.perf_counter() - t0


def _torch_cpu_standin(budget_s: float = 5.0):
    """torch's CPU einsum (BLAS DGEMM) on whole z-slabs of the workload"""
    import torch
    g = torch.Generator().manual_seed(0)
    l = torch.rand(1, 48, 48, 48, 48, generator=g, dtype=torch.float64) * 2 - 1
    r = torch.rand(1, 48, 48, 48, 48, generator=g, dtype=torch.float64) * 2 - 1
    torch.einsum(EXPR, l, r)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        torch.einsum(EXPR, l, r)
        n += 1
        el = time.perf_counter() - t0
        if el > budget_s or n >= 20:
            break
    return {"value": n * FLOPS / 64 / el / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "stand-in", "sample": f"{n} z-slab(s) (z=1, full a..f) through torch.einsum on CPU "
            "(BLAS DGEMM), the check the reference's bench_expression itself runs"}


def _cpu_baseline(budget_s: float = 15.0):
    model, cores = _lscpu()
    out = {"cpu_model": model, "host_threads": cores}
    if _ref_available():
        c, l, r, o = _ref_sample()
        times, t0 = [], time.perf_counter()
        while time.perf_counter() - t0 < budget_s and len(times) < 10:
            times.append(_time_ref_step(c, l, r, o))
        val = c.num_ops / statistics.median(times) / 1e12
        out.update({"value": val, "unit": "TFLOP/s", "cores": cores, "kind": "reference",
                    "sample": f"{len(times)} run(s) of the {SAMPLE_DESC}, {REF_DESC}; median"})
    else:
        out.update({"value": None, "unit": "TFLOP/s", "cores": cores, "kind": "reference",
                    "sample": "reference scalar library not built (no reference checkout at build time)"})
    try:
        out["stand_in_torch_cpu_einsum"] = _torch_cpu_standin()
    except Exception as e:  # a baseline, not the product: report and go on
        out["stand_in_torch_cpu_einsum"] = {"error": str(e)[:200]}
    return out


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if not _ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "reference scalar library "
                          "oracle/_ref/libref_scalar.so was not built (no reference checkout at build time)"}))
        return 0
    model, cores = _lscpu()
    c, l, r, o = _ref_sample()
    for _ in range(args.warmup):
        _time_ref_step(c, l, r, o)
    times = [_time_ref_step(c, l, r, o) for _ in range(args.steps)]
    val = c.num_ops / statistics.median(times) / 1e12
    cb = {"value": val, "unit": "TFLOP/s", "cores": cores, "kind": "reference", "cpu_model": model,
          "sample": f"each step = one run of the {SAMPLE_DESC} ({c.num_ops} flop), {REF_DESC}; "
                    "value = sample flop / median step time"}
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * statistics.mean(times), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "sampled": SAMPLE_DESC},
            "cpu_baseline": cb,
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------ GPU
def _fp64_peak(dev):
    """cuBLAS DGEMM 8192^3 (torch.matmul) best of 5, TFLOP/s"""
    import torch
    n = 8192
    a = torch.rand(n, n, device=dev, dtype=torch.float64)
    b = torch.rand(n, n, device=dev, dtype=torch.float64)
    c = torch.empty(n, n, device=dev, dtype=torch.float64)
    torch.matmul(a, b, out=c)
    best = None
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch.matmul(a, b, out=c)
        e1.record()
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    del a, b, c
    torch.cuda.empty_cache()
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


def _profile_traffic():
    """DRAM bytes of one bench launch of the DMMA kernel, from the committed ncu
    summary (a z = 8 capture scaled by the z-slabs a launch processes)"""
    import re
    f = ROOT / "profiles" / "dmma_contract_fp64_cfg5_z8.txt"
    if not f.exists():
        return None
    m = re.search(r"bench_launch_traffic_bytes:\s*([0-9.eE+]+)", f.read_text())
    return float(m.group(1)) if m else None


def run_ours(args):
    import torch
    import torch.distributed as dist
    from einsum_ir_b200 import cabi
    from einsum_ir_b200.sharded import ShardedContraction

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    if SIZES["z"] % world:
        raise SystemExit(f"z={SIZES['z']} does not split over {world} GPUs")

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

    peak = _fp64_peak(dev)
    sc = ShardedContraction(EXPR, SIZES, cabi.FP64, world, rank)
    zb = sc.layout.block
    # this rank's input blocks and the full output (every rank ends with all of it)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    l = torch.rand([zb] + [48] * 4, generator=g, device=dev, dtype=torch.float64) * 2 - 1
    r = torch.rand([zb] + [48] * 4, generator=g, device=dev, dtype=torch.float64) * 2 - 1
    out = torch.empty(sc.shape(sc.io), device=dev, dtype=torch.float64)
    gather = world > 1 and sc.bind_output(out)
    if world > 1 and not gather:
        raise SystemExit("could not map the peer outputs (CUDA IPC)")
    z0 = sc.layout.owned(rank).start
    out_blk = out[z0:z0 + zb]
    peers = sc._block_peers(out) if world > 1 else []
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    plan = sc.plan

    def step():
        if world > 1:
            plan.contract_gather(l, r, out_blk, peers, stream=sp)
        else:
            plan.contract(l, r, out_blk, stream=sp)

    # ---- device-resident timing: CUDA events around each step on the launching stream
    for _ in range(args.warmup):
        step()
    barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    launches0 = cabi.launch_count()
    barrier()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
        barrier()
    launches = cabi.launch_count() - launches0
    step_ms = sum(a.elapsed_time(b) for a, b in ev)
    step_ms_max = reduce_max(step_ms)
    value = FLOPS * args.steps / (step_ms_max * 1e-3) / 1e12

    # ---- second pass: events around the contraction kernel's own launch
    plan.profile(True)
    plan.profile_read()
    for _ in range(args.steps):
        step()
    barrier()
    kern_ms, kern_n = plan.profile_read()
    plan.profile(False)
    kern_ms_avg = reduce_max(kern_ms / max(1, kern_n))
    cabi.check_device_errors(sp)

    # ---- N > 1: the step taken apart (after the timed region, same K): the
    # contraction alone (no gather), the gather alone (this rank's finished block
    # copied to every peer, one copy stream per peer), and the overlapped step above
    breakdown = None
    if world > 1:
        def timed(fn):
            barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(args.steps):
                fn()
            b.record(stream)
            barrier()
            return reduce_max(a.elapsed_time(b) / args.steps)

        copy_streams = [torch.cuda.Stream(dev) for _ in peers]
        blk_bytes = out_blk.numel() * 8

        def gather_only():
            fork = torch.cuda.Event()
            fork.record(stream)
            for cs, p in zip(copy_streams, peers):
                cs.wait_event(fork)
                cabi.copy_to_peers(out_blk, [p], blk_bytes, stream=cs.cuda_stream)
                join = torch.cuda.Event()
                join.record(cs)
                stream.wait_event(join)

        breakdown = {"compute_only_ms": timed(lambda: plan.contract(l, r, out_blk, stream=sp)),
                     "gather_only_ms": timed(gather_only),
                     "overlapped_ms": step_ms_max / args.steps,
                     "gather_bytes_per_rank": blk_bytes * len(peers),
                     "note": "max over ranks; gather_only = cudaMemcpyAsync of the rank's block to each "
                             "peer on its own stream, no contraction"}

    # ---- correctness spot check: one z-slab of every rank's block vs torch (fp64)
    errs = []
    for rr in range(world):
        zz = sc.layout.owned(rr).start
        if rr == rank:
            ref = torch.einsum("abcd,cdef->abef", l[0], r[0])
            errs.append(float((out[zz] - ref).norm() / ref.norm()))
    rel = reduce_max(max(errs))
    gathered_finite = bool(torch.isfinite(out).all().item())

    # ---- end to end with host buffers: pinned H2D of this rank's input blocks,
    # contraction (+ gather), D2H of this rank's block of the result, pipelined
    # over groups of z-slabs on three streams. The step is bound by PCIe (the
    # H2D of 2 x the output's bytes); the first group's H2D and the last
    # group's contraction and D2H are not overlapped, so groups are small (two
    # slabs, 85 MB of output, at N = 1)
    n_groups = min(32, zb)
    gz = zb // n_groups
    from einsum_ir_b200 import binary
    g_sizes = dict(SIZES, z=gz)
    il, ir, io, names = binary.parse_binary(EXPR)
    gsz = {i: g_sizes[c] for i, c in enumerate(names)}
    gplan = cabi.ContractPlan(binary.contraction_dims(il, ir, io, gsz), cabi.FP64, cabi.FP64, cabi.FP64)
    l_h = l.cpu().pin_memory()
    r_h = r.cpu().pin_memory()
    o_h = torch.empty(out_blk.shape, dtype=torch.float64).pin_memory()
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    slab_bytes = out[0].numel() * 8

    def e2e_step():
        start = torch.cuda.Event()
        start.record(stream)
        h2d.wait_event(start)
        for gi in range(n_groups):
            sl = slice(gi * gz, (gi + 1) * gz)
            with torch.cuda.stream(h2d):
                l[sl].copy_(l_h[sl], non_blocking=True)
                r[sl].copy_(r_h[sl], non_blocking=True)
            eh = torch.cuda.Event()
            eh.record(h2d)
            stream.wait_event(eh)
            if world > 1:
                off = gi * gz * slab_bytes
                gplan.contract_gather(l[sl], r[sl], out_blk[sl], [p + off for p in peers], stream=sp)
            else:
                gplan.contract(l[sl], r[sl], out_blk[sl], stream=sp)
            ec = torch.cuda.Event()
            ec.record(stream)
            d2h.wait_event(ec)
            with torch.cuda.stream(d2h):
                o_h[sl].copy_(out_blk[sl], non_blocking=True)
        stream.wait_stream(d2h)
        stream.wait_stream(h2d)

    for _ in range(min(args.warmup, 3)):
        e2e_step()
    barrier()
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    for i in range(args.steps):
        e2e_ev[i][0].record(stream)
        e2e_step()
        e2e_ev[i][1].record(stream)
    barrier()
    e2e_ms = reduce_max(sum(a.elapsed_time(b) for a, b in e2e_ev))
    e2e_value = FLOPS * args.steps / (e2e_ms * 1e-3) / 1e12
    e2e_rel = float((o_h[0].to(dev) - out_blk[0]).abs().max().item())

    achieved = FLOPS / world / (kern_ms_avg * 1e-3) / 1e12
    line = None
    if rank == 0:
        cpu = _cpu_baseline() if world == 1 else None
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms_max / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic",
            "config": {"workload": WORKLOAD,
                       "per_rank": f"z block of {zb} slab(s); " + (
                           "eir_contract_gather: copy-engine all-gather of finished z-slabs into every "
                           "rank's full output, inside the step" if world > 1 else "whole job"),
                       "l2": "no flush: each operand (2.72 GB, or its z block) is larger than L2",
                       "plan": plan.describe(), "rel_err_vs_torch_fp64": rel,
                       "cuda_device_max_connections": os.environ.get("CUDA_DEVICE_MAX_CONNECTIONS"),
                       "gathered_output_finite": gathered_finite},
            "step_breakdown": breakdown,
            "e2e": {"value": e2e_value, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": (l.numel() + r.numel()) * 8,
                    "d2h_bytes_per_step": out_blk.numel() * 8,
                    "pipeline": f"{n_groups} groups of {gz} z-slab(s): H2D / contraction / D2H on "
                                "three streams", "d2h_check_max_abs_diff": e2e_rel},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak,
                         "traffic": (_profile_traffic() / world) if _profile_traffic() else None,
                         "traffic_source": "profiles/dmma_contract_fp64_cfg5_z8.txt (ncu z=8 capture, "
                                           "scaled by the z-slabs of this launch)",
                         "kernel": "eir::dmma_contract_kernel<%s,%s> (FP64 DMMA)" % (
                             "true" if "A=MN" in plan.describe() else "false",
                             "true" if "B=MN" in plan.describe() else "false"),
                         "peak_source": "cuBLAS DGEMM 8192^3 (torch.matmul FP64) measured in this run, best "
                                        "of 5 (MEASURED_PEAKS.json has no FP64 figure)",
                         "kernel_ms": kern_ms_avg,
                         "kernel_timing": "events around the kernel launch, second pass of the K steps"},
            "cpu_baseline": cpu,
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        sc.unbind()
        dist.barrier()  # no rank frees its output while another still maps it
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
