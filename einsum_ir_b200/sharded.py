"""Batch-sharded binary contraction across the GPUs of one node.

The output's outermost dim (a C or M dim, e.g. z in BASELINE config 5
``zabcd,zcdef->zabef``) is split into ``world`` contiguous blocks: rank r
computes block r (indices ``[r*b, (r+1)*b)``, b = size / world) with one plan
over its b slabs, reading only its blocks of the inputs, and every rank ends
with the full output. The gather has three forms:

* ``gather`` (default): ``eir_contract_gather``. The contraction writes rank
  r's block of its own full output, and the copy engines push every finished
  slab of that block into the other ranks' full outputs (mapped by the
  library's output group, eir_output_group_create, whose CUDA IPC handles
  travel over torch.distributed) while the kernel computes the next slabs. One launch covers all of the rank's slabs, so the SMs stay busy to
  the end (a launch per slab would leave the last wave of every launch partly
  empty: 324 tiles of 128 x 128 per config-5 slab on 148 SMs); the copies use
  no SM. The process should run with CUDA_DEVICE_MAX_CONNECTIONS >= 16, set
  before its CUDA context exists (``_main`` and bench.py set 32): with CUDA's
  default 8 hardware queues the waiting copy streams share queues with the
  compute stream and with one another, and at 8 GPUs the step then takes
  9.2 ms instead of 6.8 ms.
* ``nccl``: the contraction, then an in-place NCCL ``all_gather_into_tensor``
  of the rank blocks (for processes that cannot map each other's memory).
* ``fused``: ``eir_contract_peers``, the epilogue stores every output element
  into all ranks' outputs over NVLink.

One process per GPU; torch.distributed is the plumbing (handle exchange,
barriers, the NCCL fallback), the contraction, the mappings and the copies
are the C-ABI. C++ callers use einsum_ir::backend::ShardedContraction
(csrc/host/ShardedContraction.h; bench_sharded is a driver on top of it).
``python -m einsum_ir_b200.sharded`` (under torchrun) runs config 5 and prints
one JSON line on rank 0.
"""
from __future__ import annotations

import json
import os
import sys
from dataclasses import dataclass
from typing import List, Sequence

from . import binary, cabi


@dataclass
class ShardLayout:
    """Contiguous blocks of the sharded dim, one per rank, in rank order."""
    size: int      # extent of the sharded dim
    world: int

    @property
    def block(self) -> int:
        if self.size % self.world:
            raise ValueError("the sharded dim must divide into world equal blocks")
        return self.size // self.world

    def owned(self, rank: int) -> range:
        """Indices of the sharded dim rank `rank` computes."""
        b = self.block
        return range(rank * b, (rank + 1) * b)


class ShardedContraction:
    """A contraction whose output's outermost dim is sharded across ranks."""

    def __init__(self, expr: str, sizes: dict, dtype: int, world: int, rank: int,
                 dtype_comp: int = cabi.COMPUTE_DEFAULT):
        il, ir, io, names = binary.parse_binary(expr)
        self.shard_dim = io[0]
        for ids in (il, ir):
            if self.shard_dim in ids and ids[0] != self.shard_dim:
                raise ValueError("the sharded dim must be outermost in every tensor holding it")
        self.names, self.il, self.ir, self.io = names, il, ir, io
        self.sizes = {i: sizes[c] for i, c in enumerate(names)}
        self.layout = ShardLayout(self.sizes[self.shard_dim], world)
        blk = dict(self.sizes)
        blk[self.shard_dim] = self.layout.block
        self.block_sizes = blk
        dto = cabi.FP64 if dtype == cabi.FP64 else cabi.FP32
        self.plan = cabi.ContractPlan(binary.contraction_dims(il, ir, io, blk), dtype, dtype, dto,
                                      dtype_comp)
        self.world, self.rank = world, rank
        self.num_ops = self.plan.num_ops * world
        self._group = None
        self._bound = None

    def shape(self, ids: Sequence[int], block: bool = False):
        s = self.block_sizes if block else self.sizes
        return [s[i] for i in ids]

    def input_block(self, t, which: str):
        """This rank's block of a full-size input (`which` = 'left' / 'right');
        an input without the sharded dim is used whole."""
        ids = self.il if which == "left" else self.ir
        if self.shard_dim not in ids:
            return t
        rg = self.layout.owned(self.rank)
        return t[rg.start:rg.stop]

    def out_block(self, out):
        rg = self.layout.owned(self.rank)
        return out[rg.start:rg.stop]

    # ---- peer mappings of every rank's full output
    def bind_output(self, out) -> bool:
        """Maps every rank's `out` (same shape on all ranks) into this process
        through the library's output group (eir_output_group_create, CUDA IPC
        handles exchanged over torch.distributed). Collective over the default
        process group. False when some rank cannot export or map the buffers
        (then use run_nccl())."""
        import torch.distributed as dist
        self.unbind()
        if not out.is_contiguous():
            raise ValueError("bind_output: out must be contiguous")

        def allgather(data: bytes):
            parts = [None] * self.world
            dist.all_gather_object(parts, data)
            return parts
        try:
            self._group = cabi.OutputGroup(self.rank, self.world, out,
                                           allgather if self.world > 1 else (lambda d: [d]))
        except cabi.EirError:
            self._group = None
            return False
        self._bound = out.data_ptr()
        return True

    def unbind(self) -> None:
        """Closes the peer mappings (every rank, before any rank frees its output)."""
        if getattr(self, "_group", None) is not None:
            self._group.close()
        self._group, self._bound = None, None

    def _block_peers(self, out) -> List[int]:
        if self._bound != out.data_ptr():
            raise RuntimeError("bind_output(out) first")
        off = self.layout.owned(self.rank).start * out[0].numel() * out.element_size()
        return self._group.peers(off) if self.world > 1 else []

    # ---- one evaluation (asynchronous on the current stream)
    def run_gather(self, left, right, out, stream=None) -> None:
        """This rank's block into its place in `out`, copied slab by slab into
        every other rank's `out` by the copy engines (bind_output(out) first).
        The full output is complete on all ranks once every rank's stream has
        passed this call (synchronise, then a cross-rank barrier)."""
        import torch
        st = stream if stream is not None else torch.cuda.current_stream()
        self.plan.contract_gather(self.input_block(left, "left"), self.input_block(right, "right"),
                                  self.out_block(out), self._block_peers(out), stream=st.cuda_stream)

    def run_fused(self, left, right, out, stream=None) -> None:
        """This rank's block, stored by the epilogue into `out` of every rank."""
        import torch
        st = stream if stream is not None else torch.cuda.current_stream()
        self.plan.contract_peers(self.input_block(left, "left"), self.input_block(right, "right"),
                                 self.out_block(out), self._block_peers(out), stream=st.cuda_stream)

    def run_nccl(self, left, right, out, stream=None) -> None:
        """This rank's block, then an in-place NCCL all-gather of the blocks."""
        import torch
        import torch.distributed as dist
        st = stream if stream is not None else torch.cuda.current_stream()
        blk = self.out_block(out)
        self.plan.contract(self.input_block(left, "left"), self.input_block(right, "right"), blk,
                           stream=st.cuda_stream)
        if self.world > 1:
            with torch.cuda.stream(st):
                dist.all_gather_into_tensor(out.view(-1), blk.reshape(-1))


def _main() -> int:
    # the copy streams of eir_contract_gather wait on the kernel's slab
    # counters: give every stream its own hardware queue (before the CUDA
    # context exists) so a blocked wait holds back no other stream's work
    os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")
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
    z = 64
    for a in sys.argv:
        if a.startswith("--z="):
            z = int(a[4:])
    sizes = dict(z=z, a=48, b=48, c=48, d=48, e=48, f=48)
    mode = "nccl" if "--nccl" in sys.argv else ("fused" if "--fused" in sys.argv else "gather")
    sc = ShardedContraction("zabcd,zcdef->zabef", sizes, dt, world, rank, dtype_comp=comp)
    tdt = torch.float64 if dt == cabi.FP64 else torch.float32
    g = torch.Generator(device=dev).manual_seed(7)
    left = torch.rand(sc.shape(sc.il), generator=g, device=dev, dtype=tdt) * 2 - 1
    right = torch.rand(sc.shape(sc.ir), generator=g, device=dev, dtype=tdt) * 2 - 1
    out = torch.full(sc.shape(sc.io), float("nan"), device=dev, dtype=tdt)
    if mode != "nccl" and not sc.bind_output(out):
        mode = "nccl"
    step = {"fused": lambda: sc.run_fused(left, right, out),
            "gather": lambda: sc.run_gather(left, right, out),
            "nccl": lambda: sc.run_nccl(left, right, out)}[mode]
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
    cabi.check_device_errors()
    ms = e0.elapsed_time(e1) / steps
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)  # every rank has synchronised its stream
        dist.barrier()
    # check one slab computed by every rank (gathered from the others) against torch
    errs = []
    for r in range(world):
        zz = sc.layout.owned(r).start
        ref = torch.einsum("abcd,cdef->abef", left[zz], right[zz])
        errs.append(float((out[zz] - ref).norm() / ref.norm()))
    if rank == 0:
        print(json.dumps({"config": f"zabcd,zcdef->zabef z={z} a..f=48", "dtype": "fp64" if dt == cabi.FP64 else
                          ("tf32" if comp == cabi.COMPUTE_TF32 else "fp32"), "gpus": world,
                          "ms_per_eval_max_over_ranks": float(t.item()),
                          "tflops": sc.num_ops / (float(t.item()) * 1e-3) / 1e12,
                          "timed": "compute + all-gather of the full output",
                          "gather": {"fused": "fused into the epilogue (peer stores)",
                                     "gather": "copy engines, slab by slab as the kernel finishes them",
                                     "nccl": "NCCL all_gather"}[mode],
                          "plan": sc.plan.describe(),
                          "rel_err_check": max(errs)}),
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
