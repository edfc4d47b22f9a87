"""fp32 CPU reference of one (tensor-parallel) Llama decoder layer, composed
from the oracle's pinned pieces (RMSNorm, RoPE + transpose, attention,
SwiGLU) and fp32 matmuls.  Test infrastructure only.

Follows src/layers/llama_block.rs:55-65 (pre-norm block), the attention call
site src/layers/attention.rs:83-148 and the FFN src/layers/ffn.rs:47-58.
"""
from __future__ import annotations

import math

import numpy as np
import torch

import oracle


def layer_ref_fp32(x, w, cfg, n_heads_local, n_kv_local, all_reduce=lambda t: t):
    """x [B, S, d] fp32 (torch, CPU); w: this rank's weights (any dtype).
    `all_reduce` sums a torch tensor over the tensor-parallel group."""
    B, S, d = x.shape
    D = cfg.head_dim
    f = {k: v.float().cpu() for k, v in w.items()}
    xn = x.numpy()
    h, _ = oracle.rmsnorm(xn, f["norm1"].numpy(), cfg.eps)
    h = torch.from_numpy(h)
    q = (h @ f["wq"].t()).reshape(B, S, n_heads_local, D).numpy()
    k = (h @ f["wk"].t()).reshape(B, S, n_kv_local, D).numpy()
    v = (h @ f["wv"].t()).reshape(B, S, n_kv_local, D).numpy()
    ln_base = math.log(cfg.rope_base)
    q = oracle.rope_transpose(q, ln_base, cfg.rope_style)
    k = oracle.rope_transpose(k, ln_base, cfg.rope_style)
    v = np.ascontiguousarray(v.transpose(0, 2, 1, 3))
    o, _ = oracle.flash_attn2_fwd(q, k, v, 1.0 / math.sqrt(D), True)
    o = torch.from_numpy(oracle.merge_heads(o).reshape(B, S, n_heads_local * D))
    attn = o @ f["wo"].t()
    all_reduce(attn)
    h2, x2 = oracle.rmsnorm(attn.numpy(), f["norm2"].numpy(), cfg.eps, residual=xn)
    z = torch.from_numpy(h2) @ f["w_gate_up"].t()
    a = torch.from_numpy(oracle.swiglu(z.numpy()))
    ff = a @ f["w_down"].t()
    all_reduce(ff)
    return torch.from_numpy(x2) + ff


def model_ref_fp32(x, layers, norm, cfg, n_heads_local, n_kv_local, all_reduce=lambda t: t):
    """The stack (src/llama.rs:65-81 without embedding / lm_head): each layer
    in turn, then the final RMSNorm."""
    for w in layers:
        x = layer_ref_fp32(x, w, cfg, n_heads_local, n_kv_local, all_reduce)
    y, _ = oracle.rmsnorm(x.numpy(), norm.float().cpu().numpy(), cfg.eps)
    return torch.from_numpy(y)


def _heads_ref(x, w, n_heads, D, ln_base, style, rotate):
    """x [B, S, d] (torch fp32) @ w^T -> [B, n_heads, S, D] numpy, RoPE'd by position."""
    B, S, _ = x.shape
    y = (x @ w.t()).reshape(B, S, n_heads, D).numpy()
    if rotate:
        return oracle.rope_transpose(y, ln_base, style)
    return np.ascontiguousarray(y.transpose(0, 2, 1, 3))


def decoder_block_ref_fp32(tgt, enc, w, cfg, n_heads_local, n_kv_local,
                           all_reduce=lambda t: t):
    """One decoder block (src/layers/decoder_block.rs:68-81): causal
    self-attention, cross-attention on the encoder output (non-causal,
    Sq = S_t, Sk = S_e; RoPE on q and k by their own positions,
    src/layers/attention.rs:83-148) and the SwiGLU FFN, each pre-norm with a
    residual add.  tgt [B, S_t, d], enc [B, S_e, d] fp32 torch (CPU)."""
    B, S, d = tgt.shape
    D = cfg.head_dim
    f = {k: v.float().cpu() for k, v in w.items()}
    ln_base = math.log(cfg.rope_base)
    scale = 1.0 / math.sqrt(D)

    def attn(xq, xkv, p, causal):
        q = _heads_ref(xq, f[p + "q"], n_heads_local, D, ln_base, cfg.rope_style, True)
        k = _heads_ref(xkv, f[p + "k"], n_kv_local, D, ln_base, cfg.rope_style, True)
        v = _heads_ref(xkv, f[p + "v"], n_kv_local, D, ln_base, cfg.rope_style, False)
        o, _ = oracle.flash_attn2_fwd(q, k, v, scale, causal)
        out = torch.from_numpy(oracle.merge_heads(o).reshape(B, S, n_heads_local * D)) @ f[p + "o"].t()
        all_reduce(out)
        return out

    x = tgt
    h1, _ = oracle.rmsnorm(x.numpy(), f["norm1"].numpy(), cfg.eps)
    a1 = attn(torch.from_numpy(h1), torch.from_numpy(h1), "w", True)
    h2, x2 = oracle.rmsnorm(a1.numpy(), f["norm2"].numpy(), cfg.eps, residual=x.numpy())
    a2 = attn(torch.from_numpy(h2), enc, "c", False)
    h3, x3 = oracle.rmsnorm(a2.numpy(), f["norm3"].numpy(), cfg.eps, residual=x2)
    z = torch.from_numpy(h3) @ f["w_gate_up"].t()
    a = torch.from_numpy(oracle.swiglu(z.numpy()))
    ff = a @ f["w_down"].t()
    all_reduce(ff)
    return torch.from_numpy(x3) + ff


def decoder_ref_fp32(tgt, enc, blocks, norm, cfg, n_heads_local, n_kv_local,
                     all_reduce=lambda t: t):
    """Decoder blocks in turn, then the final RMSNorm (src/decoder.rs:48-53)."""
    for w in blocks:
        tgt = decoder_block_ref_fp32(tgt, enc, w, cfg, n_heads_local, n_kv_local, all_reduce)
    y, _ = oracle.rmsnorm(tgt.numpy(), norm.float().cpu().numpy(), cfg.eps)
    return torch.from_numpy(y)


def _rb(t):
    """Rounds an fp32 torch tensor or numpy array to bf16 and back (round to nearest even)."""
    if isinstance(t, np.ndarray):
        return torch.from_numpy(np.ascontiguousarray(t)).to(torch.bfloat16).float().numpy()
    return t.to(torch.bfloat16).float()


def layer_rows_ref_fp32(x, w, cfg, n_heads, n_kv, q_lo, q_hi, bf16_points=False):
    """Rows [q_lo, q_hi) of the single-rank layer's output, for full-size
    checks: K and V (and Q, for the RoPE positions) are projected for every
    token, attention and everything after it only for the sampled rows.
    x [B, S, d] fp32 torch (CPU); returns [B, q_hi - q_lo, d].

    With ``bf16_points`` the fp32 arithmetic is unchanged but the activations
    are rounded to bf16 where the fused layer stores them (h, q/k after RoPE,
    v, the attention output, o_proj's output, x2 and h2 from the fp32
    residual sum, the SwiGLU output, down_proj's output and y), so what remains
    is the kernels' own error (accumulation order, bf16 P inside attention)."""
    rb = _rb if bf16_points else (lambda t: t)
    B, S, d = x.shape
    D = cfg.head_dim
    f = {k: v.float().cpu() for k, v in w.items()}
    h, _ = oracle.rmsnorm(x.numpy(), f["norm1"].numpy(), cfg.eps)
    h = torch.from_numpy(rb(h))
    ln_base = math.log(cfg.rope_base)
    q = rb(oracle.rope_transpose((h @ f["wq"].t()).reshape(B, S, n_heads, D).numpy(), ln_base,
                                 cfg.rope_style))
    k = rb(oracle.rope_transpose((h @ f["wk"].t()).reshape(B, S, n_kv, D).numpy(), ln_base,
                                 cfg.rope_style))
    v = rb(np.ascontiguousarray((h @ f["wv"].t()).reshape(B, S, n_kv, D).numpy().transpose(0, 2, 1, 3)))
    o, _ = oracle.flash_attn2_fwd(q, k, v, 1.0 / math.sqrt(D), True, q_range=(q_lo, q_hi))
    o = rb(o[:, :, q_lo:q_hi])
    o = torch.from_numpy(np.ascontiguousarray(o.transpose(0, 2, 1, 3)).reshape(B, q_hi - q_lo,
                                                                               n_heads * D))
    attn = rb(o @ f["wo"].t())
    xr = x[:, q_lo:q_hi].contiguous().numpy()
    h2, x2 = oracle.rmsnorm(attn.numpy(), f["norm2"].numpy(), cfg.eps, residual=xr)
    h2, x2 = rb(h2), rb(x2)
    a = rb(torch.from_numpy(oracle.swiglu((torch.from_numpy(h2) @ f["w_gate_up"].t()).numpy())))
    return rb(torch.from_numpy(x2) + rb(a @ f["w_down"].t()))
