"""Tensor-parallel Llama decoder layer (prefill) over the B200 attention path.

Mirrors teenyformers' ``LlamaBlock::forward`` (src/layers/llama_block.rs:55-65)
and ``MultiHeadAttention::forward`` (src/layers/attention.rs:83-148):

    h  = RMSNorm(x)
    q, k, v = h Wq^T, h Wk^T, h Wv^T                  [B, S, H*D]
    q, k = RoPE(transpose_heads(q)), RoPE(transpose_heads(k))
    v = transpose_heads(v)
    o  = causal flash attention(q, k, v)               (GQA: Hkv KV heads)
    x2 = x + merge_heads(o) Wo^T
    y  = x2 + (SwiGLU(RMSNorm(x2) Wgu^T)) Wdown^T

The reference layer is MHA and single-device; this adds GQA and tensor
parallelism (config #5): each of the N ranks owns Hq/N query heads, Hkv/N KV
heads and d_ff/N FFN columns, so the only exchange is an all-reduce (sum) of
the o_proj and down_proj partial outputs.  The attention pieces, RoPE +
transpose, merge, RMSNorm (fused with the residual add) and SwiGLU run on
this library's sm_100a kernels; the projections are plain bf16 GEMMs
(torch.matmul -> cuBLAS).  The all-reduce is either NCCL through
torch.distributed (`all_reduce`) or, with `peer_ar` (a tp.PeerAllReduceNorm),
this library's kernel that does the all-reduce, the residual add and the
RMSNorm in one pass over NVLink peer memory.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import ops


@dataclass(frozen=True)
class LlamaLayerConfig:
    d_model: int = 4096
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    d_ff: int = 14336
    rope_base: float = 500000.0
    eps: float = 1e-5
    rope_style: int = ops.TF_ROPE_INTERLEAVED  # the reference's RopeOp (rope.rs:57-140)

    def flops(self, tokens: int, seq_len: int) -> float:
        """GEMM FLOPs plus causal attention FLOPs for `tokens` = B*S tokens."""
        d, hd = self.d_model, self.n_heads * self.head_dim
        kv = self.n_kv_heads * self.head_dim
        gemm = 2.0 * tokens * (d * hd * 2 + d * kv * 2 + d * self.d_ff * 3)
        attn = 2.0 * (tokens // seq_len) * self.n_heads * seq_len * seq_len * self.head_dim
        return gemm + attn


def shard_bounds(total: int, world: int, rank: int):
    if total % world != 0:
        raise ValueError(f"{total} does not split evenly over {world} ranks")
    per = total // world
    return rank * per, (rank + 1) * per


def init_full_weights(cfg: LlamaLayerConfig, seed: int, device, dtype=torch.bfloat16):
    """Seeded N(0, 0.02) weights of the full (unsharded) layer, generated on
    `device`; norms are 1 + N(0, 0.02).  Identical on every rank."""
    g = torch.Generator(device=device).manual_seed(seed)
    d, D = cfg.d_model, cfg.head_dim

    def w(*shape):
        return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * 0.02).to(dtype)

    return {
        "wq": w(cfg.n_heads * D, d),
        "wk": w(cfg.n_kv_heads * D, d),
        "wv": w(cfg.n_kv_heads * D, d),
        "wo": w(d, cfg.n_heads * D),
        "w_gate_up": w(2 * cfg.d_ff, d),  # [gate; up], the reference's fused layout
        "w_down": w(d, cfg.d_ff),
        "norm1": (1.0 + w(d).float()).to(dtype),
        "norm2": (1.0 + w(d).float()).to(dtype),
    }


def shard_weights(full: dict, cfg: LlamaLayerConfig, world: int, rank: int) -> dict:
    """This rank's slices: column-parallel q/k/v/gate/up, row-parallel o/down."""
    D = cfg.head_dim
    hq0, hq1 = shard_bounds(cfg.n_heads, world, rank)
    hk0, hk1 = shard_bounds(cfg.n_kv_heads, world, rank)
    f0, f1 = shard_bounds(cfg.d_ff, world, rank)
    gu = full["w_gate_up"]
    return {
        "wq": full["wq"][hq0 * D:hq1 * D].contiguous(),
        "wk": full["wk"][hk0 * D:hk1 * D].contiguous(),
        "wv": full["wv"][hk0 * D:hk1 * D].contiguous(),
        "wo": full["wo"][:, hq0 * D:hq1 * D].contiguous(),
        "w_gate_up": torch.cat([gu[f0:f1], gu[cfg.d_ff + f0:cfg.d_ff + f1]]).contiguous(),
        "w_down": full["w_down"][:, f0:f1].contiguous(),
        "norm1": full["norm1"],
        "norm2": full["norm2"],
    }


class LlamaLayerTP:
    """One decoder layer on this rank's shard; `all_reduce` sums a tensor over
    the tensor-parallel group in place (identity for one rank)."""

    def __init__(self, cfg: LlamaLayerConfig, weights: dict, world: int = 1, all_reduce=None,
                 peer_ar=None):
        if cfg.n_heads % world or cfg.n_kv_heads % world or cfg.d_ff % world:
            raise ValueError("heads and d_ff must split evenly over the ranks")
        self.cfg = cfg
        self.w = weights
        self.world = world
        self.hq = cfg.n_heads // world
        self.hkv = cfg.n_kv_heads // world
        self.ff = cfg.d_ff // world
        self.all_reduce = all_reduce or (lambda t: t)
        self.peer_ar = peer_ar
        self.scale = 1.0 / math.sqrt(cfg.head_dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        B, S, d = x.shape
        D = cfg.head_dim
        h = ops.rmsnorm(x, w["norm1"], cfg.eps)
        q = torch.matmul(h, w["wq"].t())
        k = torch.matmul(h, w["wk"].t())
        v = torch.matmul(h, w["wv"].t())
        q = ops.rope_transpose(q.view(B, S, self.hq, D), cfg.rope_base, cfg.rope_style)
        k = ops.rope_transpose(k.view(B, S, self.hkv, D), cfg.rope_base, cfg.rope_style)
        v = ops.transpose_heads(v, self.hkv)
        o, _ = ops.flash_attn2_fwd(q, k, v, self.scale, True)
        if self.peer_ar is not None:
            # partials straight into the symmetric buffer; all-reduce + residual
            # + RMSNorm in one kernel; the layer output is the second h buffer
            ar = self.peer_ar
            torch.matmul(ops.merge_heads(o), w["wo"].t(), out=ar.part.view(B, S, d))
            x2, h2 = ar(0, x, w["norm2"], cfg.eps)
            a = ops.swiglu(torch.matmul(h2.view(B, S, d), w["w_gate_up"].t()))
            torch.matmul(a, w["w_down"].t(), out=ar.part.view(B, S, d))
            out, _ = ar(1, x2)
            return out.view(B, S, d)
        attn = torch.matmul(ops.merge_heads(o), w["wo"].t())
        self.all_reduce(attn)
        h2, x2 = ops.rmsnorm(attn, w["norm2"], cfg.eps, residual=x)
        a = ops.swiglu(torch.matmul(h2, w["w_gate_up"].t()))
        f = torch.matmul(a, w["w_down"].t())
        self.all_reduce(f)
        return x2 + f
