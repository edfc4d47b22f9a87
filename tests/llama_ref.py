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
