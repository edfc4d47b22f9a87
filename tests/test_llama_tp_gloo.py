"""Tensor-parallel sharding of the Llama layer on CPU ranks (gloo, world 2):
the sharded layer with an all-reduce after o_proj and down_proj must equal the
unsharded layer.  Checks the host-side sharding (column-parallel q/k/v and
fused gate/up, row-parallel o/down) with the fp32 oracle layer."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    from llama_ref import layer_ref_fp32
    from teenyformers_b200.llama import LlamaLayerConfig, init_full_weights, shard_weights
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = LlamaLayerConfig(d_model=128, n_heads=4, n_kv_heads=2, head_dim=32, d_ff=256)
        full = init_full_weights(cfg, seed=1, device="cpu", dtype=torch.float32)
        x = torch.randn(2, 48, 128, generator=torch.Generator().manual_seed(2))
        mine = shard_weights(full, cfg, world, rank)
        y = layer_ref_fp32(x, mine, cfg, cfg.n_heads // world, cfg.n_kv_heads // world,
                           all_reduce=lambda t: dist.all_reduce(t))
        if rank == 0:
            y1 = layer_ref_fp32(x, full, cfg, cfg.n_heads, cfg.n_kv_heads)
            q.put(float((y - y1).abs().max()))
    finally:
        dist.destroy_process_group()


def test_tp2_sharded_layer_equals_full_layer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err = q.get(timeout=5)
    assert err < 1e-4, err


def test_shard_bounds_reject_uneven():
    from teenyformers_b200.llama import shard_bounds
    assert shard_bounds(32, 4, 3) == (24, 32)
    with pytest.raises(ValueError):
        shard_bounds(14, 4, 0)
