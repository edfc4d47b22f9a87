"""Tensor-parallel Llama layer over NCCL on 2 GPUs: each rank runs its shard
of the heads and FFN through this library's kernels; the all-reduced output
must match the fp32 CPU reference of the unsharded layer.  Skipped with fewer
than 2 GPUs (ranks never share a GPU)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import sys
    from datetime import timedelta

    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(__file__))
    from teenyformers_b200.llama import (LlamaLayerConfig, LlamaLayerTP, init_full_weights,
                                         shard_weights)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        cfg = LlamaLayerConfig(d_model=512, n_heads=8, n_kv_heads=2, head_dim=64, d_ff=1024)
        full = init_full_weights(cfg, seed=9, device=dev)
        x = torch.randn((2, 96, 512), generator=torch.Generator().manual_seed(4)).to(
            torch.bfloat16).to(dev)
        layer = LlamaLayerTP(cfg, shard_weights(full, cfg, world, rank), world=world,
                             all_reduce=lambda t: dist.all_reduce(t))
        y = layer.forward(x)
        torch.cuda.synchronize()
        if rank == 0:
            q.put((y.float().cpu(), x.float().cpu(), {k: v.cpu() for k, v in full.items()}))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_tp2_nccl_layer_matches_reference():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from helpers import assert_bf16_close_scaled
    from llama_ref import layer_ref_fp32
    from teenyformers_b200.llama import LlamaLayerConfig
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    y, x, full = q.get(timeout=300)
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    cfg = LlamaLayerConfig(d_model=512, n_heads=8, n_kv_heads=2, head_dim=64, d_ff=1024)
    ref = layer_ref_fp32(x, full, cfg, cfg.n_heads, cfg.n_kv_heads)
    assert_bf16_close_scaled("tp2 layer", y.numpy(), ref.numpy(), tol=3e-2)
