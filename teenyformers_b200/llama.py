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
the o_proj and down_proj partial outputs.

Default (fused) path, all on this library's sm_100a kernels:
    h        = RMSNorm(x)
    q, k, v  = one tcgen05 GEMM whose epilogue applies RoPE and writes the
               [B, H, S, 128] attention layout (transpose_heads folded in)
    o        = causal flash attention
    o_proj   = GEMM reading o in its own layout (merge_heads folded into the
               loads); with N > 1 ranks its epilogue pushes each row slice to
               the rank that owns it (the reduce-scatter, overlapped tile by
               tile), then one kernel sums the slices + residual, all-gathers
               h over NVLink and applies RMSNorm
    a        = gate/up GEMM with SwiGLU in its epilogue
    down     = GEMM; pushed like o_proj (N > 1) or with the residual add in its
               epilogue (N = 1)
The fused path needs head_dim 128 and S % 128 == 0 (and B*S a multiple of
128 * N with the peer all-reduce); other shapes, or ``fused=False``, take the
separate-kernel path: the projections are plain torch.matmul (cuBLAS) calls
followed by the separate RoPE/transpose, merge and SwiGLU kernels, and the
all-reduce is NCCL through torch.distributed (`all_reduce`) or, with
`peer_ar` (a tp.PeerAllReduceNorm), this library's all-reduce + residual +
RMSNorm kernel loading the partials over NVLink.
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
                 peer_ar=None, fused: bool = True):
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
        # the fused epilogues are built for head_dim 128; sequences must be a
        # multiple of 128 (checked per call, else the separate-kernel path runs)
        self.fused = fused and cfg.head_dim == 128
        self._tables = {}
        if self.fused:
            w = weights
            self.w_qkv = torch.cat([w["wq"], w["wk"], w["wv"]]).contiguous()
            gu = w["w_gate_up"]  # [gate shard; up shard]
            self.w_gu_blocks = ops.swiglu_weight_blocks(gu[:self.ff], gu[self.ff:])

    def _rope_table(self, S: int, device) -> torch.Tensor:
        t = self._tables.get(S)
        if t is None:
            t = ops.rope_table(S, self.cfg.head_dim, self.cfg.rope_base, device)
            self._tables[S] = t
        return t

    def _forward_fused(self, x: torch.Tensor) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        B, S, d = x.shape
        h = ops.rmsnorm(x, w["norm1"], cfg.eps)
        q, k, v = ops.linear_qkv_rope(h, self.w_qkv, self.hq, self.hkv,
                                      self._rope_table(S, x.device), cfg.rope_style)
        o, _ = ops.flash_attn2_fwd(q, k, v, self.scale, True)
        if self.peer_ar is not None:
            ar = self.peer_ar
            ops.linear_push(o, w["wo"], ar.recv_ptrs, ar.rank, ar.world, heads_seq=S)
            x2, h2 = ar(0, x, w["norm2"], cfg.eps, pushed=True)
            a = ops.linear_swiglu(h2.view(B, S, d), self.w_gu_blocks)
            ops.linear_push(a, w["w_down"], ar.recv_ptrs, ar.rank, ar.world)
            out, _ = ar(1, x2, pushed=True)
            return out.view(B, S, d)
        attn = ops.linear(o, w["wo"], heads_seq=S)
        self.all_reduce(attn)
        h2, x2 = ops.rmsnorm(attn, w["norm2"], cfg.eps, residual=x)
        a = ops.linear_swiglu(h2, self.w_gu_blocks)
        if self.world == 1:
            return ops.linear(a, w["w_down"], residual=x2)
        f = ops.linear(a, w["w_down"])
        self.all_reduce(f)
        return x2 + f

    def fused_ok(self, B: int, S: int) -> bool:
        """Whether forward() takes the fused path for a [B, S, d] input."""
        if not self.fused or S % 128:
            return False
        return self.peer_ar is None or (B * S) % (128 * self.world) == 0

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.fused_ok(x.shape[0], x.shape[1]):
            return self._forward_fused(x)
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
