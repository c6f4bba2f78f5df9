"""Multi-process logic on CPU (gloo, world size 2): the block layout of the
batch-sharded contraction and the bench's max-over-ranks timing reduction.
The per-block compute is torch.einsum on CPU here, and the gather a gloo
all-gather; on GPUs the compute is the C-ABI plan and the gather the copy
engines (einsum_ir_b200.sharded.ShardedContraction.run_gather)."""
from __future__ import annotations

import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from einsum_ir_b200.sharded import ShardLayout


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    g = torch.Generator().manual_seed(0)
    z = 6 * world
    left = torch.rand(z, 3, 2, 4, generator=g, dtype=torch.float64)   # zabc
    right = torch.rand(z, 4, 5, generator=g, dtype=torch.float64)     # zcd
    out = torch.full((z, 3, 2, 5), float("nan"), dtype=torch.float64)
    lay = ShardLayout(z, world)
    rg = lay.owned(rank)
    # this rank's block into its place, then every block into every rank's output
    out[rg.start:rg.stop] = torch.einsum("zabc,zcd->zabd", left[rg.start:rg.stop], right[rg.start:rg.stop])
    parts = [torch.empty_like(out[rg.start:rg.stop]) for _ in range(world)]
    dist.all_gather(parts, out[rg.start:rg.stop].contiguous())
    for r, p in enumerate(parts):
        o = lay.owned(r)
        out[o.start:o.stop] = p
    ref = torch.einsum("zabc,zcd->zabd", left, right)
    err = float((out - ref).abs().max())
    # bench-style timing reduction: the max over ranks
    t = torch.tensor([float(rank + 1)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    q.put((rank, err, float(t.item())))
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_layout_and_gather_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
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
        lay = ShardLayout(64, world)
        owned = [i for r in range(world) for i in lay.owned(r)]
        assert owned == list(range(64))  # contiguous blocks in rank order (NCCL all-gather order)
    with pytest.raises(ValueError):
        ShardLayout(64, 3).block
