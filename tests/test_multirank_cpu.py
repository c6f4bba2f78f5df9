"""Multi-process logic on CPU (gloo, world size 2): the block layout of the
batch-sharded contraction and the bench's max-over-ranks timing reduction.
The per-block compute is torch.einsum on CPU here; on GPUs it is the C-ABI
plan (einsum_ir_b200.sharded.ShardedContraction)."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from einsum_ir_b200.sharded import ShardLayout, run_sharded


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, chunks, q):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    g = torch.Generator().manual_seed(0)
    z = 4 * world * chunks
    left = torch.rand(z, 3, 2, 4, generator=g, dtype=torch.float64)   # zabc
    right = torch.rand(z, 4, 5, generator=g, dtype=torch.float64)     # zcd
    out = torch.full((z, 3, 2, 5), float("nan"), dtype=torch.float64)
    lay = ShardLayout(z, world, chunks)

    def compute(c, start):
        sl = slice(start, start + lay.block)
        return torch.einsum("zabc,zcd->zabd", left[sl], right[sl]).contiguous()

    def gather(dst, local):
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local)
        dst.copy_(torch.cat(parts, 0))

    run_sharded(lay, rank, compute, lambda rg: out[rg.start:rg.stop], gather)
    ref = torch.einsum("zabc,zcd->zabd", left, right)
    err = float((out - ref).abs().max())
    # bench-style timing reduction: the max over ranks
    t = torch.tensor([float(rank + 1)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    q.put((rank, err, float(t.item())))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("chunks", [1, 3])
def test_sharded_layout_and_gather_gloo(chunks):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, chunks, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, tmax in res:
        assert err == 0.0, (rank, err)
        assert tmax == float(world)


def test_shard_layout_covers_every_index_once():
    for world in (1, 2, 4, 8):
        for chunks in (1, 2, 4):
            lay = ShardLayout(64, world, chunks)
            owned = sorted(s + i for r in range(world) for s in lay.owned(r) for i in range(lay.block))
            assert owned == list(range(64))
            for c in range(chunks):
                rg = lay.gathered_range(c)
                starts = sorted(lay.owned(r)[c] for r in range(world))
                assert starts[0] == rg.start and rg.stop == starts[-1] + lay.block
