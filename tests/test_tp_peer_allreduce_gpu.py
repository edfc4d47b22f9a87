"""The fused tensor-parallel all-reduce + residual add + RMSNorm kernel over
NVLink peer memory, on 2 GPUs: against NCCL all-gather + fp32 arithmetic for
several calls in a row (epochs, both h buffers), and the whole TP layer with
the peer path against the same layer with NCCL all-reduces.  Skipped with
fewer than 2 GPUs (ranks never share a GPU)."""
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
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    out = {}
    try:
        _rank_body(rank, world, dev, out)
    except Exception as e:  # report at once instead of leaving the other rank to time out
        q.put({"error": f"rank {rank}: {e!r}"})
        raise
    finally:
        dist.destroy_process_group()
    if rank == 0:
        q.put(out)


def _rank_body(rank, world, dev, out):
    import torch.distributed as dist
    import teenyformers_b200 as tfb
    from teenyformers_b200.llama import (LlamaLayerConfig, LlamaLayerTP, init_full_weights,
                                         shard_weights)
    from teenyformers_b200.tp import PeerAllReduceNorm
    rows, cols, eps = 256, 512, 1e-5
    ar = PeerAllReduceNorm(rows, cols, device=dev)
    g = torch.Generator(device=dev).manual_seed(100)  # same on every rank
    x = torch.randn((rows, cols), generator=g, device=dev).bfloat16()
    w = (1.0 + 0.1 * torch.randn((cols,), generator=g, device=dev)).bfloat16()
    errs = []
    for call in range(3):
        gp = torch.Generator(device=dev).manual_seed(1000 * call + rank)
        ar.part.copy_(torch.randn((rows, cols), generator=gp, device=dev).bfloat16())
        slot = call % 2
        h, y = ar(slot, x if call != 1 else None, w, eps)
        parts = [torch.empty_like(ar.part) for _ in range(world)]
        dist.all_gather(parts, ar.part)
        h_ref = sum(p.float() for p in parts) + (x.float() if call != 1 else 0.0)
        y_ref = h.float() * torch.rsqrt((h.float() ** 2).mean(-1, keepdim=True) + eps) * w.float()
        torch.cuda.synchronize()
        errs.append((float((h.float() - h_ref).abs().max()),
                     float((h.float() - h_ref).abs().div(h_ref.abs().clamp(min=1)).max()),
                     float((y.float() - y_ref).abs().div(y_ref.abs().clamp(min=1)).max())))
    out["ar_errs"] = errs
    out["status"] = tfb.device_status(clear=True)
    # whole layer: peer path vs NCCL path on the same shards
    cfg = LlamaLayerConfig(d_model=512, n_heads=8, n_kv_heads=2, head_dim=64, d_ff=1024)
    full = init_full_weights(cfg, seed=9, device=dev)
    wsh = shard_weights(full, cfg, world, rank)
    xin = torch.randn((2, 64, 512), generator=torch.Generator(device=dev).manual_seed(5),
                      device=dev).bfloat16()
    ar2 = PeerAllReduceNorm(2 * 64, 512, device=dev)
    y_peer = LlamaLayerTP(cfg, wsh, world=world, peer_ar=ar2).forward(xin).clone()
    y_nccl = LlamaLayerTP(cfg, wsh, world=world,
                          all_reduce=lambda t: dist.all_reduce(t)).forward(xin)
    torch.cuda.synchronize()
    out["layer_err"] = float((y_peer.float() - y_nccl.float()).abs()
                             .div(y_nccl.float().abs().clamp(min=1)).max())
    # fused layer (QKV+RoPE epilogue, o_proj/down_proj pushing their row
    # slices to the owner ranks, local-sum all-reduce) vs the separate-kernel
    # layer with NCCL, and vs the fp32 reference of the whole layer
    from llama_ref import layer_ref_fp32
    cfg3 = LlamaLayerConfig(d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, d_ff=1024)
    full3 = init_full_weights(cfg3, seed=13, device=dev)
    wsh3 = shard_weights(full3, cfg3, world, rank)
    x3 = torch.randn((2, 128, 512), generator=torch.Generator(device=dev).manual_seed(6),
                     device=dev).bfloat16()
    ar3 = PeerAllReduceNorm(2 * 128, 512, device=dev)
    fused = LlamaLayerTP(cfg3, wsh3, world=world, peer_ar=ar3)
    assert fused.fused_ok(2, 128)
    ys = [fused.forward(x3).clone() for _ in range(3)]  # repeated calls: epochs, reuse
    y_ref3 = LlamaLayerTP(cfg3, wsh3, world=world, fused=False,
                          all_reduce=lambda t: dist.all_reduce(t)).forward(x3)
    torch.cuda.synchronize()
    out["fused_err"] = float((ys[-1].float() - y_ref3.float()).abs()
                             .div(y_ref3.float().abs().clamp(min=1)).max())
    out["fused_repeat"] = all(torch.equal(ys[0], y) for y in ys[1:])
    if rank == 0:
        ref = layer_ref_fp32(x3.float().cpu(), full3, cfg3, 4, 2)
        out["fused_ref_err"] = float((ys[-1].float().cpu() - ref).abs()
                                     .div(ref.abs().clamp(min=1)).max())
    out["status2"] = tfb.device_status(clear=True)
    dist.barrier()


def test_peer_allreduce_residual_rmsnorm_2gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    env_nvls = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
        for p in procs:
            p.start()
        out = q.get(timeout=300)
        for p in procs:
            p.join(60 if "error" in out else 120)
            if p.is_alive():
                p.terminate()
                p.join(30)
    finally:
        if env_nvls is None:
            os.environ.pop("NCCL_NVLS_ENABLE", None)
        else:
            os.environ["NCCL_NVLS_ENABLE"] = env_nvls
    assert "error" not in out, out.get("error")
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert out["status"] == 0
    for abs_err, rel_h, rel_y in out["ar_errs"]:
        # h: fp32 sum rounded once to bf16 (2^-9 relative); y from that h
        assert rel_h <= 1e-2 and rel_y <= 2e-2, out["ar_errs"]
    assert out["layer_err"] <= 3e-2, out["layer_err"]
    assert out["status2"] == 0
    assert out["fused_err"] <= 3e-2, out["fused_err"]
    assert out["fused_ref_err"] <= 3e-2, out["fused_ref_err"]
    assert out["fused_repeat"], "fused TP layer must be repeatable"
