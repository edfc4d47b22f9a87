"""The multi-GPU path shards attention over batch x heads with no collective
on the data path.  These world-size-2 gloo tests (CPU) check the host logic:
the shards cover every head exactly once, per-rank results assemble into the
single-rank result bit for bit, and timings reduce to the max over ranks."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench
import oracle


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, H, S, D = 2, 4, 48, 32
        g = torch.Generator().manual_seed(0)
        qkv = [torch.randn((B * H, S, D), generator=g) for _ in range(3)]
        lo, hi = bench.shard_heads(B * H, world, rank)
        o, lse = oracle.flash_attn2_fwd(*(t[lo:hi].numpy() for t in qkv), D ** -0.5, True)
        gathered = [torch.zeros((B * H // world, S, D)) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(o[0]))
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            full, _ = oracle.flash_attn2_fwd(*(x.numpy() for x in qkv), D ** -0.5, True)
            q.put((bool(np.array_equal(torch.cat(gathered).numpy(), full[0])), float(t.item())))
    finally:
        dist.destroy_process_group()


def test_shard_heads_partition():
    for world in (1, 2, 4, 8):
        spans = [bench.shard_heads(256, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 256
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        bench.shard_heads(10, 4, 0)


def test_two_rank_gloo_sharded_attention_matches_single_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    same, tmax = q.get(timeout=5)
    assert same, "sharded results differ from the single-rank result"
    assert tmax == 2.0
