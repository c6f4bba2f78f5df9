"""Batch-sharded binary contraction across the GPUs of one node.

The output's outermost dim (a C or M dim, e.g. z in BASELINE config 5
``zabcd,zcdef->zabef``) is split into ``world * chunks`` blocks. Rank r owns
blocks ``c * world + r`` (c = 0..chunks-1), so block c of all ranks together is
one contiguous slice of the output: after computing its block c a rank
all-gathers it straight into that slice (``all_gather_into_tensor``, NCCL over
NVLink), on a communication stream, while it computes block c+1. The
contraction itself is the C-ABI plan of one block (one process per GPU;
torch.distributed is only the plumbing).

Fused gather (``bind_output`` + ``run_fused``): every rank maps the other
ranks' output buffers into its process (CUDA IPC, handles exchanged over
torch.distributed) and runs its slab of the contraction with
``eir_contract_peers``: the contraction's epilogue stores each output tile
into all ranks' outputs over NVLink while the next tiles compute, so no
collective competes with the persistent contraction kernel for SMs (with a
separate NCCL all-gather the two serialise: the contraction kernel occupies
every SM). The NCCL path stays for processes that cannot map each other's
memory.

``python -m einsum_ir_b200.sharded`` (under torchrun) runs config 5 and prints
one JSON line per rank 0 (``--nccl``: the NCCL all-gather path).
"""
from __future__ import annotations

import json
import os
import sys
from dataclasses import dataclass
from typing import Callable, List, Sequence

from . import binary, cabi


@dataclass
class ShardLayout:
    """Which blocks of the sharded dim a rank owns and where they land."""
    size: int      # extent of the sharded dim
    world: int
    chunks: int

    @property
    def block(self) -> int:
        if self.size % (self.world * self.chunks):
            raise ValueError("sharded dim must divide into world * chunks blocks")
        return self.size // (self.world * self.chunks)

    def owned(self, rank: int) -> List[int]:
        """Start index (in the sharded dim) of each block rank `rank` computes, in order."""
        return [(c * self.world + rank) * self.block for c in range(self.chunks)]

    def gathered_range(self, c: int) -> range:
        """Indices of the sharded dim filled by the all-gather of block round c."""
        b = self.block
        return range(c * self.world * b, (c + 1) * self.world * b)


def run_sharded(layout: ShardLayout, rank: int, compute: Callable[[int, int], object],
                out_rows: Callable[[range], object], gather: Callable[[object, object], None],
                wait: Callable[[], None] | None = None) -> None:
    """Drives the block rounds: compute(c, start) returns the local block
    result, out_rows(range) the destination slice, gather(dst, src) enqueues the
    all-gather (which may overlap the next compute); wait() drains it."""
    for c, start in enumerate(layout.owned(rank)):
        local = compute(c, start)
        gather(out_rows(layout.gathered_range(c)), local)
    if wait is not None:
        wait()


class ShardedContraction:
    """Config-5 style contraction with the sharded dim outermost in every tensor."""

    def __init__(self, expr: str, sizes: dict, dtype: int, world: int, rank: int, chunks: int = 4,
                 dtype_comp: int = cabi.COMPUTE_DEFAULT):
        il, ir, io, names = binary.parse_binary(expr)
        self.shard_dim = io[0]
        for ids in (il, ir):
            if self.shard_dim in ids and ids[0] != self.shard_dim:
                raise ValueError("the sharded dim must be outermost in every tensor holding it")
        self.names, self.il, self.ir, self.io = names, il, ir, io
        self.sizes = {i: sizes[c] for i, c in enumerate(names)}
        self.layout = ShardLayout(self.sizes[self.shard_dim], world, chunks)
        blk = dict(self.sizes)
        blk[self.shard_dim] = self.layout.block
        self.block_sizes = blk
        dto = cabi.FP64 if dtype == cabi.FP64 else cabi.FP32
        self.plan = cabi.ContractPlan(binary.contraction_dims(il, ir, io, blk), dtype, dtype, dto,
                                      dtype_comp)
        self.world, self.rank = world, rank
        self.num_ops = self.plan.num_ops * world * chunks
        self._peer_ptrs: List[int] = []
        self._peer_bases: List[int] = []
        self._bound = None

    def shape(self, ids: Sequence[int], block: bool = False):
        s = self.block_sizes if block else self.sizes
        return [s[i] for i in ids]

    def run(self, left, right, out, comm_stream=None):
        """left/right: this rank's full-size inputs (only its blocks are read);
        out: full output on every rank (filled by the all-gathers)."""
        import torch
        import torch.distributed as dist
        lay = self.layout
        compute_stream = torch.cuda.current_stream()
        comm = comm_stream or torch.cuda.Stream()
        locals_ = []

        def compute(c, start):
            blk = torch.empty(self.shape(self.io, True), dtype=out.dtype, device=out.device)
            lsl = left[start:start + lay.block] if self.shard_dim in self.il else left
            rsl = right[start:start + lay.block] if self.shard_dim in self.ir else right
            self.plan.contract(lsl, rsl, blk, stream=compute_stream.cuda_stream)
            ev = torch.cuda.Event()
            ev.record(compute_stream)
            locals_.append((blk, ev))
            return len(locals_) - 1

        def gather(dst, idx):
            blk, ev = locals_[idx]
            comm.wait_event(ev)
            blk.record_stream(comm)  # the caching allocator must not reuse it before the gather ends
            with torch.cuda.stream(comm):
                if self.world > 1:
                    dist.all_gather_into_tensor(dst, blk)
                else:
                    dst.copy_(blk)

        run_sharded(lay, self.rank, compute, lambda rg: out[rg.start:rg.stop], gather,
                    lambda: compute_stream.wait_stream(comm))

    # ---- fused gather: the epilogue writes every rank's output
    def bind_output(self, out) -> bool:
        """Maps every rank's `out` (same shape on all ranks) into this process.
        Collective over the default process group. False when some rank
        cannot export or map the buffers (then use run())."""
        import torch.distributed as dist
        self.unbind()
        if self.world == 1:
            self._bound = out.data_ptr()
            return True
        try:
            handle, off = cabi.ipc_get_handle(out)
            mine = (handle, off, True)
        except cabi.EirError:
            mine = (b"", 0, False)
        objs = [None] * self.world
        dist.all_gather_object(objs, mine)
        ok = all(o[2] for o in objs)
        ptrs, bases = [], []
        if ok:
            try:
                for r in range(self.world):
                    if r == self.rank:
                        continue
                    ptr, base = cabi.ipc_open_handle(objs[r][0], objs[r][1])
                    ptrs.append(ptr)
                    bases.append(base)
            except cabi.EirError:
                ok = False
        flags = [None] * self.world
        dist.all_gather_object(flags, ok)
        if not all(flags):
            for b in bases:
                cabi.ipc_close_handle(b)
            return False
        self._peer_ptrs, self._peer_bases, self._bound = ptrs, bases, out.data_ptr()
        return True

    def unbind(self) -> None:
        """Closes the peer mappings (every rank, before any rank frees its output)."""
        for b in self._peer_bases:
            cabi.ipc_close_handle(b)
        self._peer_ptrs, self._peer_bases, self._bound = [], [], None

    def run_ce(self, left, right, out, comm_streams=None) -> None:
        """This rank's blocks, each computed into its final place in the local
        `out` and then copied by the copy engines into every other rank's
        `out` (bind_output(out) first) while the next block computes: the
        gather takes no SM from the contraction kernel. The copy to each peer
        runs on a stream of its own (`comm_streams`, one per peer), so the
        copies of one block proceed in parallel on several copy engines
        instead of one after another. The output is complete on all ranks
        once every rank's stream has passed this call (synchronise, then a
        cross-rank barrier, before reading)."""
        import torch
        if self._bound != out.data_ptr():
            raise RuntimeError("run_ce: bind_output(out) first")
        if not out.is_contiguous():
            raise ValueError("run_ce: out must be contiguous")
        lay = self.layout
        compute = torch.cuda.current_stream()
        comm = list(comm_streams) if comm_streams else []
        while len(comm) < len(self._peer_ptrs):
            comm.append(torch.cuda.Stream())
        row_bytes = out[0].numel() * out.element_size()
        for start in lay.owned(self.rank):
            lsl = left[start:start + lay.block] if self.shard_dim in self.il else left
            rsl = right[start:start + lay.block] if self.shard_dim in self.ir else right
            dst = out[start:start + lay.block]
            self.plan.contract(lsl, rsl, dst, stream=compute.cuda_stream)
            if self._peer_ptrs:
                ev = torch.cuda.Event()
                ev.record(compute)
                off = start * row_bytes
                for peer, st in zip(self._peer_ptrs, comm):
                    st.wait_event(ev)
                    cabi.copy_to_peers(dst, [peer + off], lay.block * row_bytes, stream=st.cuda_stream)
        for st in comm[:len(self._peer_ptrs)]:
            compute.wait_stream(st)

    def run_fused(self, left, right, out) -> None:
        """This rank's blocks, each stored by the epilogue into `out` of every
        rank at its final place (bind_output(out) first). The output is
        complete on all ranks once every rank's stream has passed this call
        (synchronise, then a cross-rank barrier, before reading it)."""
        import torch
        if self._bound != out.data_ptr():
            raise RuntimeError("run_fused: bind_output(out) first")
        lay = self.layout
        stream = torch.cuda.current_stream().cuda_stream
        if not out.is_contiguous():
            raise ValueError("run_fused: out must be contiguous")
        row_bytes = out[0].numel() * out.element_size()
        for start in lay.owned(self.rank):
            lsl = left[start:start + lay.block] if self.shard_dim in self.il else left
            rsl = right[start:start + lay.block] if self.shard_dim in self.ir else right
            dst = out[start:start + lay.block]
            off = start * row_bytes  # the block's byte offset, the same in every rank's output
            self.plan.contract_peers(lsl, rsl, dst, [p + off for p in self._peer_ptrs], stream=stream)


def _main() -> int:
    import time
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    dt = cabi.FP64 if "--fp32" not in sys.argv else cabi.FP32
    comp = cabi.COMPUTE_TF32 if "--tf32" in sys.argv else cabi.COMPUTE_DEFAULT
    sizes = dict(z=64, a=48, b=48, c=48, d=48, e=48, f=48)
    mode = "nccl" if "--nccl" in sys.argv else ("fused" if "--fused" in sys.argv else "ce")
    z = sizes["z"]
    chunks = {"fused": 1, "nccl": 4 if world < 8 else 2, "ce": max(1, min(8, z // world))}[mode]
    sc = ShardedContraction("zabcd,zcdef->zabef", sizes, dt, world, rank, chunks=chunks, dtype_comp=comp)
    tdt = torch.float64 if dt == cabi.FP64 else torch.float32
    g = torch.Generator(device=dev).manual_seed(7)
    left = torch.rand(sc.shape(sc.il), generator=g, device=dev, dtype=tdt)
    right = torch.rand(sc.shape(sc.ir), generator=g, device=dev, dtype=tdt)
    out = torch.empty(sc.shape(sc.io), device=dev, dtype=tdt)
    if mode != "nccl" and not sc.bind_output(out):
        mode = "nccl"
        sc = ShardedContraction("zabcd,zcdef->zabef", sizes, dt, world, rank,
                                chunks=4 if world < 8 else 2, dtype_comp=comp)
    comm = torch.cuda.Stream()
    comm_streams = [torch.cuda.Stream() for _ in range(max(0, world - 1))]
    step = {"fused": lambda: sc.run_fused(left, right, out),
            "ce": lambda: sc.run_ce(left, right, out, comm_streams),
            "nccl": lambda: sc.run(left, right, out, comm)}[mode]
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = 3
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)  # every rank has synchronised its stream
        dist.barrier()
    # spot check one gathered block of another rank against torch
    zz = sc.layout.owned((rank + 1) % world)[0]
    ref = torch.einsum("abcd,cdef->abef", left[zz], right[zz])
    rel = float((out[zz] - ref).norm() / ref.norm())
    if rank == 0:
        print(json.dumps({"config": "zabcd,zcdef->zabef z=64 a..f=48", "dtype": "fp64" if dt == cabi.FP64 else
                          ("tf32" if comp == cabi.COMPUTE_TF32 else "fp32"), "gpus": world,
                          "ms_per_eval_max_over_ranks": float(t.item()),
                          "tflops": sc.num_ops / (float(t.item()) * 1e-3) / 1e12,
                          "timed": "compute + all-gather of the full output",
                          "gather": {"fused": "fused into the epilogue (peer stores)",
                                     "ce": "copy engines (peer copies overlapping the next block)",
                                     "nccl": "NCCL all_gather"}[mode],
                          "rel_err_check": rel}),
              flush=True)
    if world > 1:
        dist.barrier()
        if mode != "nccl":
            sc.unbind()
        dist.barrier()  # no rank frees its output while another still maps it
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(_main())
