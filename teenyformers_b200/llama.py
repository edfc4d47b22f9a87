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
separate-kernel path, still entirely on this library's kernels: the
projections run on the same tcgen05 GEMM without epilogue fusion, followed by
the separate RoPE/transpose, merge and SwiGLU kernels, and the all-reduce is
NCCL through torch.distributed (`all_reduce`) or, with `peer_ar` (a
tp.PeerAllReduceNorm), this library's all-reduce + residual + RMSNorm kernel
loading the partials over NVLink.  ``projections="cublas"`` swaps the
separate path's projections for torch.matmul; it exists only as a named
comparison arm for the benchmark and is never chosen implicitly.

``LlamaModelTP`` stacks the layers and applies the final RMSNorm
(``Llama::forward``, src/llama.rs:65-81, without the token embedding and the
weight-tied lm_head, which are not on the attention path).
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
                 peer_ar=None, fused: bool = True, projections: str = "ours"):
        if cfg.n_heads % world or cfg.n_kv_heads % world or cfg.d_ff % world:
            raise ValueError("heads and d_ff must split evenly over the ranks")
        if projections not in ("ours", "cublas"):
            raise ValueError("projections must be 'ours' or 'cublas'")
        if projections == "cublas" and fused:
            raise ValueError("projections='cublas' is a comparison arm of the separate-kernel "
                             "path: pass fused=False with it")
        self.projections = projections
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

    def _mm(self, a: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None,
            residual: torch.Tensor | None = None) -> torch.Tensor:
        """a @ weight.T (+ residual): this library's GEMM, or cuBLAS for the
        explicitly requested comparison arm."""
        if self.projections == "ours":
            return ops.linear(a, weight, out=out, residual=residual)
        y = torch.matmul(a, weight.t(), out=out)
        return y if residual is None else y.add_(residual)

    def _o_proj(self, o: torch.Tensor, S: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """merge_heads(o) @ Wo^T; head_dim 128 and S % 128 == 0 read o in its own
        layout (the GEMM's heads-layout A loads whole 128-row blocks of a head)."""
        if self.projections == "ours" and self.cfg.head_dim == 128 and S % 128 == 0:
            return ops.linear(o, self.w["wo"], out=out, heads_seq=S)
        return self._mm(ops.merge_heads(o), self.w["wo"], out=out)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.fused_ok(x.shape[0], x.shape[1]):
            return self._forward_fused(x)
        cfg, w = self.cfg, self.w
        B, S, d = x.shape
        D = cfg.head_dim
        h = ops.rmsnorm(x, w["norm1"], cfg.eps)
        q = self._mm(h, w["wq"])
        k = self._mm(h, w["wk"])
        v = self._mm(h, w["wv"])
        q = ops.rope_transpose(q.view(B, S, self.hq, D), cfg.rope_base, cfg.rope_style)
        k = ops.rope_transpose(k.view(B, S, self.hkv, D), cfg.rope_base, cfg.rope_style)
        v = ops.transpose_heads(v, self.hkv)
        o, _ = ops.flash_attn2_fwd(q, k, v, self.scale, True)
        if self.peer_ar is not None:
            # partials straight into the symmetric buffer; all-reduce + residual
            # + RMSNorm in one kernel; the layer output is the second h buffer
            ar = self.peer_ar
            self._o_proj(o, S, out=ar.part.view(B, S, d))
            x2, h2 = ar(0, x, w["norm2"], cfg.eps)
            a = ops.swiglu(self._mm(h2.view(B, S, d), w["w_gate_up"]))
            self._mm(a, w["w_down"], out=ar.part.view(B, S, d))
            out, _ = ar(1, x2)
            return out.view(B, S, d)
        attn = self._o_proj(o, S)
        self.all_reduce(attn)
        h2, x2 = ops.rmsnorm(attn, w["norm2"], cfg.eps, residual=x)
        a = ops.swiglu(self._mm(h2, w["w_gate_up"]))
        if self.world == 1:
            return self._mm(a, w["w_down"], residual=x2)
        f = self._mm(a, w["w_down"])
        self.all_reduce(f)
        return x2 + f


class LlamaModelTP:
    """The Llama decoder stack on this rank's shards: ``n_layers`` pre-norm
    blocks, then the final RMSNorm (src/llama.rs:65-81).  The token embedding
    and the weight-tied lm_head around it are outside the attention path and
    are not built; ``forward`` maps hidden states [B, S, d] to the normalised
    hidden states the lm_head would read.

    ``layer_weights`` holds one shard_weights(...) dict per layer; every other
    argument is passed to each LlamaLayerTP.  With ``peer_ar`` each layer's
    output is a view of the all-reduce's second h buffer, which the next layer
    reads as its input before its own all-reduce writes that buffer again."""

    def __init__(self, cfg: LlamaLayerConfig, layer_weights: list, norm_weight: torch.Tensor,
                 **layer_kwargs):
        if not layer_weights:
            raise ValueError("the stack needs at least one layer")
        self.cfg = cfg
        self.layers = [LlamaLayerTP(cfg, w, **layer_kwargs) for w in layer_weights]
        self.norm = norm_weight

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for layer in self.layers:
            x = layer.forward(x)
        return ops.rmsnorm(x, self.norm, self.cfg.eps)


def init_model_weights(cfg: LlamaLayerConfig, n_layers: int, seed: int, device,
                       dtype=torch.bfloat16):
    """Full (unsharded) weights of an n_layers stack: one init_full_weights
    dict per layer (seeds seed, seed+1, ...) and the final norm's weight."""
    layers = [init_full_weights(cfg, seed + i, device, dtype) for i in range(n_layers)]
    g = torch.Generator(device=device).manual_seed(seed + n_layers)
    norm = (1.0 + 0.02 * torch.randn(cfg.d_model, generator=g, device=device,
                                      dtype=torch.float32)).to(dtype)
    return layers, norm
