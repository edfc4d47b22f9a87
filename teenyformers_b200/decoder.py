"""Transformer decoder block and stack over the B200 attention path.

Mirrors teenyformers' ``DecoderBlock::forward`` (src/layers/decoder_block.rs:
68-81) and ``Decoder::forward`` (src/decoder.rs:48-53):

    x2  = tgt + SelfAttn(RMSNorm(tgt))                causal
    x3  = x2 + CrossAttn(RMSNorm(x2), enc)           queries from the decoder,
                                                      keys / values from the
                                                      encoder output, no mask
    out = x3 + FFN(RMSNorm(x3))                       SwiGLU
    Decoder: blocks in turn, then the final RMSNorm.

Cross-attention is the attention op's non-causal caller with Sq != Sk
(``FlashAttn2Op``, flash_attn2.rs:393-429): q [B, Hq, S_t, D] against k, v
[B, Hkv, S_e, D].  As in ``MultiHeadAttention::forward``
(src/layers/attention.rs:83-148) RoPE rotates q and k by their own sequence
positions (0..S_t-1 and 0..S_e-1), and the encoder output is projected
without a norm.  The reference block is MHA; n_kv_heads < n_heads (GQA) is
this build's extension, as in the Llama layer.

Every step runs on this library's kernels: RMSNorm with the residual add
fused, the tcgen05 GEMM (the self-attention projections through the QKV
epilogue that applies RoPE and writes the attention layout when head_dim is
128 and S_t % 128 == 0; otherwise GEMM + the RoPE/transpose kernel), the
flash-attention forward, o_proj reading the attention output in its own
layout, and the gate/up GEMM with SwiGLU in its epilogue.  Tensor parallel
over N ranks as in the Llama layer: Hq/N and Hkv/N heads and d_ff/N FFN
columns per rank, with ``all_reduce`` (sum, e.g. NCCL) after each of the
three row-parallel projections.
"""
from __future__ import annotations

import math

import torch

from . import ops
from .llama import LlamaLayerConfig, shard_bounds


def init_decoder_block_weights(cfg: LlamaLayerConfig, seed: int, device,
                               dtype=torch.bfloat16) -> dict:
    """Seeded N(0, 0.02) weights of one full decoder block (norms 1 + N(0, 0.02)):
    self-attention wq/wk/wv/wo, cross-attention cq/ck/cv/co, FFN w_gate_up/w_down."""
    g = torch.Generator(device=device).manual_seed(seed)
    d, D = cfg.d_model, cfg.head_dim

    def w(*shape):
        return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * 0.02).to(dtype)

    out = {}
    for p in ("w", "c"):
        out[p + "q"] = w(cfg.n_heads * D, d)
        out[p + "k"] = w(cfg.n_kv_heads * D, d)
        out[p + "v"] = w(cfg.n_kv_heads * D, d)
        out[p + "o"] = w(d, cfg.n_heads * D)
    out["w_gate_up"] = w(2 * cfg.d_ff, d)
    out["w_down"] = w(d, cfg.d_ff)
    for n in ("norm1", "norm2", "norm3"):
        out[n] = (1.0 + w(d).float()).to(dtype)
    return out


def shard_decoder_block_weights(full: dict, cfg: LlamaLayerConfig, world: int,
                                rank: int) -> dict:
    """This rank's slices: column-parallel q/k/v (both attentions) and gate/up,
    row-parallel o (both attentions) and down."""
    D = cfg.head_dim
    hq0, hq1 = shard_bounds(cfg.n_heads, world, rank)
    hk0, hk1 = shard_bounds(cfg.n_kv_heads, world, rank)
    f0, f1 = shard_bounds(cfg.d_ff, world, rank)
    gu = full["w_gate_up"]
    out = {}
    for p in ("w", "c"):
        out[p + "q"] = full[p + "q"][hq0 * D:hq1 * D].contiguous()
        out[p + "k"] = full[p + "k"][hk0 * D:hk1 * D].contiguous()
        out[p + "v"] = full[p + "v"][hk0 * D:hk1 * D].contiguous()
        out[p + "o"] = full[p + "o"][:, hq0 * D:hq1 * D].contiguous()
    out["w_gate_up"] = torch.cat([gu[f0:f1], gu[cfg.d_ff + f0:cfg.d_ff + f1]]).contiguous()
    out["w_down"] = full["w_down"][:, f0:f1].contiguous()
    for n in ("norm1", "norm2", "norm3"):
        out[n] = full[n]
    return out


class DecoderBlockTP:
    """One pre-norm decoder block on this rank's shard; ``all_reduce`` sums a
    tensor over the tensor-parallel group in place (identity for one rank)."""

    def __init__(self, cfg: LlamaLayerConfig, weights: dict, world: int = 1, all_reduce=None):
        if cfg.n_heads % world or cfg.n_kv_heads % world or cfg.d_ff % world:
            raise ValueError("heads and d_ff must split evenly over the ranks")
        self.cfg = cfg
        self.w = weights
        self.world = world
        self.hq = cfg.n_heads // world
        self.hkv = cfg.n_kv_heads // world
        self.ff = cfg.d_ff // world
        self.all_reduce = all_reduce or (lambda t: t)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        w = weights
        self.w_qkv = torch.cat([w["wq"], w["wk"], w["wv"]]).contiguous()
        gu = w["w_gate_up"]
        self.w_gu_blocks = (ops.swiglu_weight_blocks(gu[:self.ff], gu[self.ff:])
                            if self.ff % 128 == 0 else None)
        self._tables = {}

    def _rope_table(self, S: int, device) -> torch.Tensor:
        t = self._tables.get(S)
        if t is None:
            t = ops.rope_table(S, self.cfg.head_dim, self.cfg.rope_base, device)
            self._tables[S] = t
        return t

    def _heads(self, x: torch.Tensor, weight: torch.Tensor, n_heads: int, rotate: bool):
        """[B, S, d] -> x W^T as [B, n_heads, S, D], RoPE'd by position if `rotate`."""
        B, S, _ = x.shape
        y = ops.linear(x, weight).view(B, S, n_heads, self.cfg.head_dim)
        if rotate:
            return ops.rope_transpose(y, self.cfg.rope_base, self.cfg.rope_style)
        return ops.transpose_heads(y.view(B, S, n_heads * self.cfg.head_dim), n_heads)

    def _o_proj(self, o: torch.Tensor, weight: torch.Tensor, S: int,
                residual: torch.Tensor | None = None) -> torch.Tensor:
        if self.cfg.head_dim == 128 and S % 128 == 0:  # o read in its own layout
            return ops.linear(o, weight, heads_seq=S, residual=residual)
        return ops.linear(ops.merge_heads(o), weight, residual=residual)

    def _sub_out(self, o: torch.Tensor, weight: torch.Tensor, S: int,
                 residual: torch.Tensor) -> torch.Tensor:
        """residual + merge_heads(o) W^T: the residual add rides in the GEMM's
        epilogue on one rank, after the all-reduce otherwise."""
        if self.world == 1:
            return self._o_proj(o, weight, S, residual=residual)
        part = self._o_proj(o, weight, S)
        self.all_reduce(part)
        return residual + part

    def forward(self, tgt: torch.Tensor, enc: torch.Tensor) -> torch.Tensor:
        """tgt [B, S_t, d], enc [B, S_e, d] -> out [B, S_t, d]."""
        cfg, w = self.cfg, self.w
        S = tgt.shape[1]
        # causal self-attention
        h1 = ops.rmsnorm(tgt, w["norm1"], cfg.eps)
        if cfg.head_dim == 128 and S % 128 == 0:
            q, k, v = ops.linear_qkv_rope(h1, self.w_qkv, self.hq, self.hkv,
                                          self._rope_table(S, tgt.device), cfg.rope_style)
        else:
            q = self._heads(h1, w["wq"], self.hq, True)
            k = self._heads(h1, w["wk"], self.hkv, True)
            v = self._heads(h1, w["wv"], self.hkv, False)
        o, _ = ops.flash_attn2_fwd(q, k, v, self.scale, True)
        x2 = self._sub_out(o, w["wo"], S, tgt)
        # cross-attention: queries from the decoder, keys / values from the encoder
        h2 = ops.rmsnorm(x2, w["norm2"], cfg.eps)
        q = self._heads(h2, w["cq"], self.hq, True)
        k = self._heads(enc, w["ck"], self.hkv, True)
        v = self._heads(enc, w["cv"], self.hkv, False)
        o, _ = ops.flash_attn2_fwd(q, k, v, self.scale, False)
        x3 = self._sub_out(o, w["co"], S, x2)
        # SwiGLU FFN
        h3 = ops.rmsnorm(x3, w["norm3"], cfg.eps)
        if self.w_gu_blocks is not None:
            a = ops.linear_swiglu(h3, self.w_gu_blocks)
        else:
            a = ops.swiglu(ops.linear(h3, w["w_gate_up"]))
        if self.world == 1:
            return ops.linear(a, w["w_down"], residual=x3)
        f = ops.linear(a, w["w_down"])
        self.all_reduce(f)
        return x3 + f


class DecoderTP:
    """Decoder blocks in turn, then the final RMSNorm (src/decoder.rs:48-53)."""

    def __init__(self, cfg: LlamaLayerConfig, block_weights: list, norm_weight: torch.Tensor,
                 world: int = 1, all_reduce=None):
        if not block_weights:
            raise ValueError("the decoder needs at least one block")
        self.cfg = cfg
        self.blocks = [DecoderBlockTP(cfg, w, world, all_reduce) for w in block_weights]
        self.norm = norm_weight

    def forward(self, tgt: torch.Tensor, enc: torch.Tensor) -> torch.Tensor:
        for block in self.blocks:
            tgt = block.forward(tgt, enc)
        return ops.rmsnorm(tgt, self.norm, self.cfg.eps)
