#!/usr/bin/env python3
"""Benchmark of the attention hot path on B200 (one process per GPU).

Headline workload (BASELINE config #3): causal flash-attention-2 forward +
backward, bf16, B=8, H=32, S=4096, D=128.  A step is one forward and one
backward over this rank's share of the B*H heads (strong scaling: the 256
heads are split across the N ranks with no collective on the data path).
Also measured: RoPE + head transpose (config #2, [4,2048,32,128] bf16) GB/s;
GQA causal forward (config #4, B16 Hq64 Hkv8 S8192, KV groups split across the
ranks, no collective); the tensor-parallel Llama-3-8B-shaped decoder layer
prefill (config #5, B4 S4096, heads and FFN split across the ranks with an
NCCL all-reduce after o_proj and down_proj).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Rank 0 prints one JSON line.  Timing: CUDA events on the launching stream,
barrier + synchronize on both sides, max over ranks.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "FA2 fwd/bwd TFLOP/s (bf16 causal S4096 D128) at 1/2/4/8 B200; RoPE GB/s"
CFG3 = dict(batch=8, heads=32, seq=4096, head_dim=128, causal=True)
CFG2 = dict(batch=4, seq=2048, heads=32, head_dim=128, rope_base=10000.0)
CFG4 = dict(batch=16, heads_q=64, heads_kv=8, seq=8192, head_dim=128)
CFG_DEC = dict(batch=64, heads_q=32, heads_kv=8, head_dim=128, cap=4096, min_len=1024, n_q=1)
CFG5 = dict(batch=4, seq=4096, d_model=4096, heads=32, kv_heads=8, head_dim=128, d_ff=14336,
            rope_base=500000.0, eps=1e-5)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def shard_heads(bh: int, world: int, rank: int):
    """Contiguous range of the B*H heads owned by `rank` (no collective on the
    data path: attention is independent per head)."""
    if bh % world != 0:
        raise ValueError(f"{bh} heads do not split evenly over {world} ranks")
    per = bh // world
    return rank * per, (rank + 1) * per


def attn_flops(B, H, S, D, causal=True):
    """FA2 convention: fwd 4*B*H*S^2*D (x1/2 causal), bwd = 2.5 x fwd."""
    fwd = 4.0 * B * H * S * S * D * (0.5 if causal else 1.0)
    return fwd, 2.5 * fwd


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def load_traffic():
    """DRAM bytes per launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return {}


# ----------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = set(gpu_indices)
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in self.gpus:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() in ("active", "1"):
                        reasons.add(n)
        finally:
            os.unlink(self.path)
        if not sm:
            return None
        top = max(sm)
        loaded = [s for s in sm if s >= 0.5 * top] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- CPU legs
def cpu_attention_sample(threads=None):
    """Oracle (fp32 restatement of the reference kernels) on one (b,h) slice
    of config #3 at full S: causal fwd + bwd.  Returns (seconds, flops)."""
    import numpy as np
    import oracle

    if threads:
        oracle.set_threads(threads)
    S, D = CFG3["seq"], CFG3["head_dim"]
    rng = np.random.default_rng(42)
    q, k, v, do = (rng.standard_normal((1, 1, S, D)).astype(np.float32) for _ in range(4))
    scale = D ** -0.5
    t0 = time.perf_counter()
    o, lse = oracle.flash_attn2_fwd(q, k, v, scale, True)
    oracle.flash_attn2_bwd(q, k, v, o, do, lse, scale, True)
    dt = time.perf_counter() - t0
    f, b = attn_flops(1, 1, S, D, True)
    return dt, f + b


def reference_arm(args, rank, world):
    """--impl reference: the reference's algorithm on the host cores.  The
    reference itself (Rust DSL + absent compiler) cannot be built here, so
    this times the oracle port; rank 0 only."""
    if rank != 0:
        return
    import oracle

    threads = oracle.max_threads()
    for _ in range(max(args.warmup, 0) and 1):
        cpu_attention_sample()
    times = []
    flops = 0.0
    for _ in range(args.steps):
        dt, flops = cpu_attention_sample()
        times.append(dt)
    mean = sum(times) / len(times)
    value = flops / mean / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1))", "impl": "reference",
        "config": {"workload": "config#3 FA2 fwd+bwd causal B8 H32 S4096 D128",
                   "sample_per_step": "1 of 256 (b,h) slices at full S=4096"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": "1 of 256 (b,h) slices of config #3 (fwd+bwd) per step; "
                                   "throughput is per-slice FLOP / time (linear in B*H)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU legs
def _timed(stream, n, fn):
    import torch
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(n):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n


def gqa_leg(args, dev, world, rank, barrier, max_over_ranks, peaks):
    """Config #4: causal GQA forward, the B*Hkv = 128 KV groups (each with its
    8 query heads) split evenly over the ranks; no collective."""
    import torch

    import teenyformers_b200 as tfb
    B, Hq, Hkv, S, D = (CFG4[k] for k in ("batch", "heads_q", "heads_kv", "seq", "head_dim"))
    if Hkv % world:
        return {"skipped": f"{Hkv} KV heads do not split over {world} ranks"}
    hq_l, hkv_l = Hq // world, Hkv // world
    g = torch.Generator(device=dev).manual_seed(4242 + rank)
    q = torch.randn((B, hq_l, S, D), generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn((B, hkv_l, S, D), generator=g, device=dev, dtype=torch.bfloat16)
    v = torch.randn((B, hkv_l, S, D), generator=g, device=dev, dtype=torch.bfloat16)
    o = torch.empty_like(q)
    lse = torch.empty((B, hq_l, S), device=dev, dtype=torch.float32)
    scale = D ** -0.5
    run = lambda: tfb.flash_attn2_fwd(q, k, v, scale, True, out=o, lse=lse)
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        run()
    n = max(3, min(args.steps, 10))
    barrier()
    torch.cuda.synchronize()
    ms = max_over_ranks(_timed(stream, n, run))
    barrier()
    flops = 2.0 * B * Hq * S * S * D  # causal: 4*B*H*S^2*D / 2
    tf = flops / (ms * 1e-3) / 1e12
    del q, k, v, o, lse
    return {"tflops": tf, "tflops_per_gpu": tf / world, "ms_per_step": ms, "steps": n,
            "frac_of_peak": tf / world / peaks["bf16_tflops"],
            "frac_of_sustained": tf / world / peaks["bf16_tflops_sustained"],
            "peak_used": "bf16_tflops (burst): the timed region is well under a second",
            "launches": n,
            "workload": f"config#4 GQA causal fwd B{B} Hq{Hq} Hkv{Hkv} S{S} D{D}; "
                        f"{hkv_l} KV heads x {B} batches per rank; Q is "
                        f"{B * hq_l * S * D * 2 / 2**30:.1f} GiB per rank (> L2)"}


def decode_leg(args, dev, world, rank, barrier, max_over_ranks, peaks):
    """KV-cache decode (the next caller of the attention op after prefill):
    Llama-3-8B attention shape, B=64 sequences with cached lengths uniform in
    [1024, 4096], one new token each; sequences split evenly over the ranks.
    HBM-bound: every cached K/V byte is read once."""
    import numpy as np
    import torch

    import teenyformers_b200 as tfb
    c = CFG_DEC
    if c["batch"] % world:
        return {"skipped": f"{c['batch']} sequences do not split over {world} ranks"}
    B = c["batch"] // world
    Hq, Hkv, D, cap, n_q = c["heads_q"], c["heads_kv"], c["head_dim"], c["cap"], c["n_q"]
    lens_all = np.random.default_rng(7).integers(c["min_len"], cap + 1, size=c["batch"])
    lens = lens_all[rank * B:(rank + 1) * B]
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    q = torch.randn((B, Hq, n_q, D), generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn((B, Hkv, cap, D), generator=g, device=dev, dtype=torch.bfloat16)
    v = torch.randn((B, Hkv, cap, D), generator=g, device=dev, dtype=torch.bfloat16)
    seq = torch.tensor(lens, dtype=torch.int32, device=dev)
    o = torch.empty_like(q)
    lse = torch.empty((B, Hq, n_q), dtype=torch.float32, device=dev)
    ws = tfb.decode_workspace(q, Hkv, cap)
    scale = D ** -0.5
    run = lambda: tfb.flash_attn2_decode(q, k, v, seq, scale, out=o, lse=lse, workspace=ws)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 3)):
        run()
    n = max(args.steps, 20)
    graph = torch.cuda.CUDAGraph()  # ~0.1 ms launches: time them without host gaps
    with torch.cuda.graph(graph):
        for _ in range(n):
            run()
    graph.replay()
    barrier()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    graph.replay()
    b.record(stream)
    torch.cuda.synchronize()
    barrier()
    us = max_over_ranks(a.elapsed_time(b) / n * 1e3)
    del graph
    kv_bytes = int(2 * Hkv * D * 2 * int(lens_all.sum()))
    qo_bytes = 2 * c["batch"] * Hq * n_q * D * 2
    gbs = (kv_bytes + qo_bytes) / (us * 1e-6) / 1e9
    del q, k, v, o
    return {"gbs": gbs, "gbs_per_gpu": gbs / world, "us_per_step": us, "steps": n,
            "bytes_per_step": kv_bytes + qo_bytes,
            "frac_of_hbm": gbs / world / peaks["hbm_gbs"],
            "peak_used": "hbm_gbs (measured copy bandwidth)",
            "workload": f"decode B{c['batch']} Hq{Hq} Hkv{Hkv} D{D} n_q{n_q}, cached lengths "
                        f"uniform in [{c['min_len']}, {cap}] (seed 7), {B} sequences per rank; "
                        f"K/V cache {B * Hkv * cap * D * 4 / 2**30:.2f} GiB per rank (> L2); "
                        f"{n} launches in one CUDA graph replay"}


def tfb_status() -> int:
    """The library's device status word (0 unless a bounded device wait expired); cleared."""
    import teenyformers_b200 as tfb
    return tfb.device_status(clear=True)


def llama_leg(args, dev, world, rank, barrier, max_over_ranks, peaks):
    """Config #5: one Llama-3-8B-shaped decoder layer prefill, tensor-parallel
    over the ranks (all-reduce after o_proj and down_proj)."""
    import torch
    import torch.distributed as dist

    from teenyformers_b200.llama import (LlamaLayerConfig, LlamaLayerTP, init_full_weights,
                                         shard_weights)
    c = CFG5
    cfg = LlamaLayerConfig(d_model=c["d_model"], n_heads=c["heads"], n_kv_heads=c["kv_heads"],
                           head_dim=c["head_dim"], d_ff=c["d_ff"], rope_base=c["rope_base"],
                           eps=c["eps"])
    if cfg.n_kv_heads % world:
        return {"skipped": f"{cfg.n_kv_heads} KV heads do not split over {world} ranks"}
    full = init_full_weights(cfg, seed=5, device=dev)
    w = shard_weights(full, cfg, world, rank)
    del full
    g = torch.Generator(device=dev).manual_seed(55)  # same activations on every rank
    x = torch.randn((c["batch"], c["seq"], c["d_model"]), generator=g, device=dev,
                    dtype=torch.bfloat16)
    stream = torch.cuda.current_stream(dev)
    tokens = c["batch"] * c["seq"]
    flops = cfg.flops(tokens, c["seq"])
    n = max(3, min(args.steps, 10))

    def measure_interleaved(layers, rounds=3):
        """Median over `rounds` of each layer's mean step time; the variants
        alternate within every round so they see the same clock / power state
        (the GPU runs at its power cap here and its clocks drift over seconds)."""
        for layer in layers:
            for _ in range(args.warmup):
                layer.forward(x)
        times = [[] for _ in layers]
        for _ in range(rounds):
            for i, layer in enumerate(layers):
                barrier()
                torch.cuda.synchronize()
                times[i].append(max_over_ranks(_timed(stream, n, lambda: layer.forward(x))))
        barrier()
        return [sorted(t)[len(t) // 2] for t in times]

    res = {}
    if world > 1:
        from teenyformers_b200.tp import PeerAllReduceNorm
        peer = PeerAllReduceNorm(tokens, c["d_model"], device=dev)
        layer = LlamaLayerTP(cfg, w, world=world, peer_ar=peer)
        assert layer.fused_ok(c["batch"], c["seq"])
        ms, ms_peer, ms_nccl = measure_interleaved([
            layer, LlamaLayerTP(cfg, w, world=world, peer_ar=peer, fused=False),
            LlamaLayerTP(cfg, w, world=world, fused=False, projections="cublas",
                         all_reduce=lambda t: dist.all_reduce(t))])
        res["cublas_nccl_ms_per_step"] = ms_nccl
        res["cublas_nccl_tflops"] = flops / (ms_nccl * 1e-3) / 1e12
        res["unfused_peer_ms_per_step"] = ms_peer
        collective = ("o_proj / down_proj GEMMs push their row slices to the owner ranks over "
                      "NVLink (reduce-scatter overlapped with the GEMM), then one kernel sums the "
                      "slices + residual, all-gathers h with peer stores and applies RMSNorm; "
                      "comparison arms: unfused_peer_* = this library's GEMM without epilogue "
                      "fusion + separate kernels + the peer all-reduce kernel; cublas_nccl_* = "
                      "cuBLAS projections + separate kernels + NCCL all-reduces")
        launches = 8
    else:
        layer = LlamaLayerTP(cfg, w, world=world)
        assert layer.fused_ok(c["batch"], c["seq"])
        ms, ms_unfused, ms_cublas = measure_interleaved([
            layer, LlamaLayerTP(cfg, w, world=world, fused=False),
            LlamaLayerTP(cfg, w, world=world, fused=False, projections="cublas")])
        res["unfused_ms_per_step"] = ms_unfused
        res["unfused_tflops"] = flops / (ms_unfused * 1e-3) / 1e12
        res["cublas_ms_per_step"] = ms_cublas
        res["cublas_tflops"] = flops / (ms_cublas * 1e-3) / 1e12
        collective = ("no collective at TP x1; comparison arms: unfused_* = this library's "
                      "GEMM without epilogue fusion + separate RoPE/transpose, merge, SwiGLU "
                      "kernels; cublas_* = the same with cuBLAS projections")
        launches = 7
    tf = flops / (ms * 1e-3) / 1e12
    del w, x, layer
    res["device_status"] = tfb_status()
    res.update({"tflops": tf, "tokens_per_s": tokens / (ms * 1e-3), "ms_per_step": ms,
                "steps": n, "timing": "median of 3 rounds, variants interleaved within a round",
                "flops_per_step": flops,
                "frac_of_peak": tf / world / peaks["bf16_tflops"],
                "frac_of_sustained": tf / world / peaks["bf16_tflops_sustained"],
                "peak_used": "bf16_tflops (burst): each timed region is well under a second",
                "launches_per_step_ours": launches,
                "workload": f"config#5 Llama-3-8B-shaped layer prefill B{c['batch']} S{c['seq']} "
                            f"d{c['d_model']} H{c['heads']}/{c['kv_heads']} ff{c['d_ff']}, "
                            f"TP x{world}; every kernel from this library: RMSNorm, QKV GEMM "
                            "with RoPE + head transpose in its epilogue, causal attention, "
                            "o_proj GEMM reading the attention layout, gate/up GEMM with "
                            "SwiGLU epilogue, down GEMM; " + collective})
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-chunks", type=int, default=8,
                    help="head chunks the end-to-end leg pipelines over")
    ap.add_argument("--no-rope", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-gqa", action="store_true")
    ap.add_argument("--no-llama", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--small", action="store_true",
                    help="profiling case: 2 of 8 batches (inputs still > L2)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        reference_arm(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    import teenyformers_b200 as tfb

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    peaks, peak_src = load_peaks()
    B, H, S, D = CFG3["batch"], CFG3["heads"], CFG3["seq"], CFG3["head_dim"]
    if args.small:
        B = 2
    BH = B * H
    head_lo, head_hi = shard_heads(BH, world, rank)
    bh_local = head_hi - head_lo
    scale = D ** -0.5
    fwd_flops_total, bwd_flops_total = attn_flops(B, H, S, D, True)
    fwd_flops_rank = fwd_flops_total / world
    bwd_flops_rank = bwd_flops_total / world

    # ---- inputs: this rank's heads, seeded by global head range ----
    g = torch.Generator(device=dev).manual_seed(42 + rank)
    shape = (1, bh_local, S, D)
    q, k, v, do = (torch.randn(shape, generator=g, device=dev, dtype=torch.bfloat16)
                   for _ in range(4))
    o = torch.empty_like(q)
    lse = torch.empty((1, bh_local, S), device=dev, dtype=torch.float32)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ws = tfb.bwd_workspace(q)
    step_bytes = 8 * q.numel() * 2 + ws.numel()  # the tensors one step touches, + workspace
    stream = torch.cuda.current_stream(dev)

    def step():
        tfb.flash_attn2_fwd(q, k, v, scale, True, out=o, lse=lse)
        tfb.flash_attn2_bwd(q, k, v, o, lse, do, scale, True, workspace=ws, grads=(dq, dk, dv))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if tfb.device_status(clear=True) != 0:
        raise RuntimeError("device-side wait timed out during warm-up")

    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = [int(x) for x in vis.split(",")] if vis else list(range(max(world, 1)))
    sampler = ClockSampler(phys[:world] if world > 1 else [phys[local_rank] if vis else local_rank])
    if rank == 0:
        sampler.start()
        time.sleep(0.3)

    # ---- timed region: K steps of fwd + bwd ----
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        tfb.flash_attn2_fwd(q, k, v, scale, True, out=o, lse=lse)
        ev[i][1].record(stream)
        tfb.flash_attn2_bwd(q, k, v, o, lse, do, scale, True, workspace=ws, grads=(dq, dk, dv))
        ev[i][2].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    total_ms = max_over_ranks(t_start.elapsed_time(t_end))
    fwd_ms = max_over_ranks(sum(e[0].elapsed_time(e[1]) for e in ev) / args.steps)
    bwd_ms = max_over_ranks(sum(e[1].elapsed_time(e[2]) for e in ev) / args.steps)
    ms_per_step = total_ms / args.steps
    value = (fwd_flops_total + bwd_flops_total) / (ms_per_step * 1e-3) / 1e12
    fwd_tflops_rank = fwd_flops_rank / (fwd_ms * 1e-3) / 1e12
    bwd_tflops_rank = bwd_flops_rank / (bwd_ms * 1e-3) / 1e12
    status = tfb.device_status(clear=True)

    # ---- RoPE + transpose leg (config #2, every rank runs the full config) ----
    # The tensor-bound steps above leave the GPU at its power cap with lowered
    # SM clocks, which stretch the fixed per-launch work of a ~24 us kernel; the
    # memory-bound legs start after a second of idle, by which the clocks recover.
    if not (args.no_rope and args.no_decode):
        torch.cuda.synchronize()
        time.sleep(1.0)
    rope = None
    if not args.no_rope:
        rb, rs, rh, rd = CFG2["batch"], CFG2["seq"], CFG2["heads"], CFG2["head_dim"]
        n_bufs = 4  # 4 x 128 MiB of in+out rotates through the 126 MB L2
        xs = [torch.randn((rb, rs, rh, rd), generator=g, device=dev, dtype=torch.bfloat16)
              for _ in range(n_bufs)]
        ys = [torch.empty((rb, rh, rs, rd), device=dev, dtype=torch.bfloat16)
              for _ in range(n_bufs)]
        n_rope = max(args.steps, 20) * n_bufs

        def time_style(style):
            for i in range(max(args.warmup, 3) * n_bufs):
                tfb.rope_transpose(xs[i % n_bufs], CFG2["rope_base"], style, out=ys[i % n_bufs])
            # Capture the launches in a CUDA graph and time one replay: a ~20 us
            # kernel launched through Python is otherwise timed together with the
            # host's launch gaps.
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(n_rope):
                    tfb.rope_transpose(xs[i % n_bufs], CFG2["rope_base"], style,
                                       out=ys[i % n_bufs])
            graph.replay()
            barrier()
            torch.cuda.synchronize()
            ra = torch.cuda.Event(enable_timing=True)
            rb_ = torch.cuda.Event(enable_timing=True)
            ra.record(stream)
            graph.replay()
            rb_.record(stream)
            torch.cuda.synchronize()
            barrier()
            us = max_over_ranks(ra.elapsed_time(rb_) / n_rope * 1e3)
            del graph
            return us

        rope_bytes = 2 * rb * rs * rh * rd * 2
        rope_us = time_style(tfb.TF_ROPE_ROTATE_HALF)
        inter_us = time_style(tfb.TF_ROPE_INTERLEAVED)
        rope_gbs = rope_bytes / (rope_us * 1e-6) / 1e9
        inter_gbs = rope_bytes / (inter_us * 1e-6) / 1e9
        rope = {"gbs_per_gpu": rope_gbs, "us_per_launch": rope_us, "bytes_per_launch": rope_bytes,
                "frac_of_hbm": rope_gbs / peaks["hbm_gbs"],
                "peak_used": "hbm_gbs (measured copy bandwidth)",
                "interleaved": {"gbs_per_gpu": inter_gbs, "us_per_launch": inter_us,
                                "frac_of_hbm": inter_gbs / peaks["hbm_gbs"],
                                "style": "interleaved pairs (2k, 2k+1), the reference's "
                                         "rope.rs pairing"},
                "workload": "config#2 x[4,2048,32,128] bf16 -> RoPE(rotate-half, theta 1e4) -> "
                            "[4,32,2048,128]; 4 rotating buffer sets (512 MiB) so reads miss L2; "
                            f"{n_rope} launches in one CUDA graph replay per style, after 1 s "
                            "idle (clocks recover from the power cap of the fwd+bwd steps)"}
        del xs, ys

    # the memory-bound decode leg goes before the long tensor-bound legs, which leave the
    # GPU at its power cap with lowered SM clocks
    decode = None if args.no_decode else decode_leg(args, dev, world, rank, barrier,
                                                    max_over_ranks, peaks)
    gqa = None if args.no_gqa else gqa_leg(args, dev, world, rank, barrier, max_over_ranks,
                                           peaks)
    llama = None if args.no_llama else llama_leg(args, dev, world, rank, barrier,
                                                 max_over_ranks, peaks)

    clocks = sampler.stop() if rank == 0 else None

    # ---- end to end through the public API, host buffers ----
    # Pinned host Q, K, V, dO in, O, LSE, dQ, dK, dV out, every step.  The
    # heads go in chunks over three streams (copy in / compute / copy out) so
    # PCIe transfers in both directions overlap each other and the kernels,
    # as a caller of flash_attn2_fwd/bwd would pipeline them; consecutive steps
    # stream back to back (step i+1's uploads overlap step i's downloads), each
    # chunk's buffers reused once the previous step is done with them.  Host
    # and device staging are chunk-major: a chunk's Q, K, V, dO are one
    # contiguous block (and its O, dQ, dK, dV another, LSE a third), so a chunk
    # crosses PCIe in one copy per direction plus the LSE copy (many small
    # copies cost PCIe time: 144 copies of 7.4 MB each way took 28.8 ms against
    # 22.2 ms for one 1 GiB copy each way).  The API is called per chunk on
    # [1, heads, S, D] views of those blocks.  The timed region runs from the
    # first upload of the first timed step to the last download of the last
    # one; e2e = that time / steps.
    e2e = None
    if not args.no_e2e:
        n_e2e = max(3, min(args.steps, 10))
        n_chunks = max(1, min(args.e2e_chunks, bh_local))
        while bh_local % n_chunks:
            n_chunks -= 1
        hc = bh_local // n_chunks
        blk = (n_chunks, 4, hc, S, D)
        in_d = torch.empty(blk, dtype=torch.bfloat16, device=dev)
        out_d = torch.empty(blk, dtype=torch.bfloat16, device=dev)
        lse_d = torch.empty((n_chunks, hc, S), dtype=torch.float32, device=dev)
        in_h = torch.empty(blk, dtype=torch.bfloat16, pin_memory=True)
        for t_i, src in enumerate((q, k, v, do)):  # the same inputs as the device-timed run
            in_h[:, t_i].copy_(src[0].reshape(n_chunks, hc, S, D).cpu())
        out_h = torch.empty(blk, dtype=torch.bfloat16, pin_memory=True)
        lse_h = torch.empty((n_chunks, hc, S), dtype=torch.float32, pin_memory=True)
        s_in, s_cmp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
        ws_c = tfb.bwd_workspace(in_d[0, 0][None])
        done_cmp = [None] * n_chunks  # per chunk: the last step's kernels finished
        done_out = [None] * n_chunks  # per chunk: the last step's downloads finished

        def e2e_step():
            for c in range(n_chunks):
                with torch.cuda.stream(s_in):
                    if done_cmp[c] is not None:
                        s_in.wait_event(done_cmp[c])  # inputs of chunk c no longer read
                    in_d[c].copy_(in_h[c], non_blocking=True)
                    e_in = torch.cuda.Event()
                    e_in.record(s_in)
                with torch.cuda.stream(s_cmp):
                    s_cmp.wait_event(e_in)
                    if done_out[c] is not None:
                        s_cmp.wait_event(done_out[c])  # outputs of chunk c downloaded
                    qc, kc, vc, doc = (in_d[c, t_i][None] for t_i in range(4))
                    oc, dqc, dkc, dvc = (out_d[c, t_i][None] for t_i in range(4))
                    lc = lse_d[c][None]
                    tfb.flash_attn2_fwd(qc, kc, vc, scale, True, out=oc, lse=lc)
                    tfb.flash_attn2_bwd(qc, kc, vc, oc, lc, doc, scale, True, workspace=ws_c,
                                        grads=(dqc, dkc, dvc))
                    done_cmp[c] = torch.cuda.Event()
                    done_cmp[c].record(s_cmp)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(done_cmp[c])
                    out_h[c].copy_(out_d[c], non_blocking=True)
                    lse_h[c].copy_(lse_d[c], non_blocking=True)
                    done_out[c] = torch.cuda.Event()
                    done_out[c].record(s_out)

        e2e_step()
        torch.cuda.synchronize()
        barrier()
        ev_start = torch.cuda.Event(enable_timing=True)
        ev_end = torch.cuda.Event(enable_timing=True)
        ev_start.record(s_in)
        for _ in range(n_e2e):
            e2e_step()
        s_out.wait_stream(s_in)
        ev_end.record(s_out)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(ev_start.elapsed_time(ev_end) / n_e2e)
        h2d = in_h.numel() * in_h.element_size() * world
        d2h = (out_h.numel() * out_h.element_size() + lse_h.numel() * lse_h.element_size()) * world
        e2e = {"value": (fwd_flops_total + bwd_flops_total) / (e2e_ms * 1e-3) / 1e12,
               "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": e2e_ms, "steps": n_e2e, "chunks": n_chunks,
               "path": "pinned host Q,K,V,dO -> flash_attn2_fwd/bwd (C ABI) on "
                       f"{n_chunks} head chunks, uploads / kernels / downloads on three "
                       "streams, steps streamed back to back, chunk-major staging (one "
                       "copy per chunk and direction + LSE) -> pinned host O,LSE,dQ,dK,dV"}
        del in_d, out_d, lse_d

    # ---- CPU baseline (rank 0, N=1 only) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle

        cpu_attention_sample()  # warm caches / thread pool
        dts = []
        fl = 0.0
        for _ in range(2):
            dt, fl = cpu_attention_sample()
            dts.append(dt)
        dt = min(dts)
        cpu = {"value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": oracle.max_threads(),
               "kind": "port",
               "sample": "1 of 256 (b,h) slices of config #3 at full S=4096 (causal fwd+bwd, "
                         f"{dt:.2f} s), best of 2; throughput linear in B*H"}

    if rank == 0:
        traffic = load_traffic()
        # the committed traffic is for config #3's 256 heads on one GPU; a rank's share
        # (or the --small case) moves bytes in proportion to its heads
        t_scale = bh_local / 256.0

        def t_of(key):
            v = traffic.get(key)
            return None if v is None else v * t_scale
        # every kernel here is timed in a region far shorter than a second, so the
        # burst GEMM figure is the denominator; the sustained one is reported beside it
        bf16_peak = peaks["bf16_tflops"]
        fwd_ach = fwd_tflops_rank
        bwd_ach = bwd_tflops_rank
        dominant = "fa_bwd" if bwd_ms >= fwd_ms else "fa_fwd"
        roof_fwd = {"kernel": "fa_fwd_sm100_kernel<128>", "bound": "tensor", "achieved": fwd_ach,
                    "peak": bf16_peak, "unit": "TFLOP/s", "frac": fwd_ach / bf16_peak,
                    "frac_of_sustained": fwd_ach / peaks["bf16_tflops_sustained"],
                    "traffic": t_of("fa_fwd"),
                    "flops_per_launch": fwd_flops_rank, "ms_per_launch": fwd_ms}
        roof_bwd = {"kernel": "fa_bwd (prep + fused dK/dV/dQ + dQ convert kernels, one C-ABI call)",
                    "bound": "tensor", "achieved": bwd_ach, "peak": bf16_peak,
                    "unit": "TFLOP/s", "frac": bwd_ach / bf16_peak,
                    "frac_of_sustained": bwd_ach / peaks["bf16_tflops_sustained"],
                    "traffic": t_of("fa_bwd"),
                    "flops_per_launch": bwd_flops_rank, "ms_per_launch": bwd_ms}
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1), torch generator on device)",
            "config": {"workload": f"config#3 FA2 fwd+bwd causal B{B} H{H} S{S} D{D}"
                                   + (" (small profiling case)" if args.small else ""),
                       "batch": B, "heads": H, "seq_len": S, "head_dim": D,
                       "heads_per_gpu": bh_local, "parallelism": f"bh-shard x{world}",
                       "l2": "inputs larger than L2: each step reads and writes "
                             f"{step_bytes / 2**20:.0f} MiB per GPU (Q,K,V,dO,O,dQ,dK,dV of "
                             f"{q.numel() * 2 / 2**20:.0f} MiB each + the fp32 dQ accumulator) "
                             "against a 126 MB L2, so each step starts with the previous "
                             "step's inputs evicted"},
            "fwd_tflops": fwd_flops_total / (fwd_ms * 1e-3) / 1e12,
            "bwd_tflops": bwd_flops_total / (bwd_ms * 1e-3) / 1e12,
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
            "roofline": roof_bwd if dominant == "fa_bwd" else roof_fwd,
            "roofline_all": [roof_fwd, roof_bwd],
            "peak_source": f"{peak_src} (MEASURED_PEAKS.json: roofline.peak = bf16 burst "
                           f"{peaks['bf16_tflops']} TFLOP/s, the figure for kernels timed in "
                           f"sub-second regions; sustained {peaks['bf16_tflops_sustained']} "
                           f"reported as frac_of_sustained; HBM {peaks['hbm_gbs']} GB/s)",
            "rope": rope,
            "gqa_fwd": gqa,
            "llama_layer": llama,
            "decode": decode,
            "rope_gbs": rope["gbs_per_gpu"] if rope else None,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": 4 * args.steps,
            "gpu_launches_note": "fwd 1 + bwd 3 (prep, fused dK/dV/dQ, dQ convert) per timed step of the "
                                 "headline loop; the rope/gqa/llama legs count their own",
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
