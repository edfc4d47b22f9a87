#!/usr/bin/env python3
"""Regenerates the committed golden fixtures under tests/golden/.

Two kinds of fixture:

1. ``rope_ref/``, ``swiglu_ref/``, ``fused_add_rmsnorm_ref/`` -- the
   reference's OWN golden vectors, copied byte for byte from the teenyformers
   checkout (``tests/fixtures/{rope,swiglu,fused_add_rmsnorm}/``, produced there
   by ``tests/fixtures/generate.py:43-128`` and checked by
   ``tests/kernel_execution.rs:63-215`` at abs-tol 1e-4).  They pin the
   oracle's interleaved RoPE, SwiGLU and fused add + RMSNorm.  Needs the
   reference checkout: ``--reference /path/to/teenyformers``.

2. ``attn_*.npz`` -- attention known-answer vectors computed by torch in
   float64 with the reference kernel's semantics (top-left causal mask,
   natural-log LSE of the scaled scores, flash_attn2.rs:77-125; gradients of
   flash_attn2.rs:155-202 via autograd).  The reference's attention kernels
   cannot be run anywhere here (Rust DSL + absent compiler), so these are an
   independent second witness, not reference outputs.  Inputs are
   torch.manual_seed(42) N(0,1), stored in the fixture.

Usage: python tests/golden/make_golden.py --reference <teenyformers checkout>
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, B, Hq, Hkv, Sq, Sk, D, causal)
ATTN_CASES = [
    ("attn_cfg1_causal_b1h4s128d64", 1, 4, 4, 128, 128, 64, True),  # BASELINE config #1
    ("attn_causal_ragged_b2h2s77d64", 2, 2, 2, 77, 77, 64, True),
    ("attn_cross_b1h2q40k72d32", 1, 2, 2, 40, 72, 32, False),
    ("attn_causal_topleft_b1h2q96k40d64", 1, 2, 2, 96, 40, 64, True),
    ("attn_gqa_causal_b1h4kv2s64d128", 1, 4, 2, 64, 64, 128, True),
]


def attention_fp64(q, k, v, do, scale, causal):
    """Reference semantics in float64: returns o, lse, dq, dk, dv."""
    B, Hq, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    G = Hq // Hkv
    q = q.double().requires_grad_(True)
    k = k.double().requires_grad_(True)
    v = v.double().requires_grad_(True)
    ke = k.repeat_interleave(G, dim=1)
    ve = v.repeat_interleave(G, dim=1)
    s = torch.einsum("bhqd,bhkd->bhqk", q, ke) * scale
    if causal:
        mask = torch.ones(Sq, Sk, dtype=torch.bool).triu(diagonal=1)  # k > q masked
        s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse[..., None])
    o = torch.einsum("bhqk,bhkd->bhqd", p, ve)
    o.backward(do.double())
    return (o.detach(), lse.detach(), q.grad.detach(), k.grad.detach(), v.grad.detach())


def make_attn():
    torch.manual_seed(42)
    for name, B, Hq, Hkv, Sq, Sk, D, causal in ATTN_CASES:
        q = torch.randn(B, Hq, Sq, D)
        k = torch.randn(B, Hkv, Sk, D)
        v = torch.randn(B, Hkv, Sk, D)
        do = torch.randn(B, Hq, Sq, D)
        scale = 1.0 / float(np.sqrt(D))
        o, lse, dq, dk, dv = attention_fp64(q, k, v, do, scale, causal)
        np.savez(
            os.path.join(HERE, name + ".npz"),
            q=q.numpy(), k=k.numpy(), v=v.numpy(), do=do.numpy(),
            o=o.float().numpy(), lse=lse.float().numpy(),
            dq=dq.float().numpy(), dk=dk.float().numpy(), dv=dv.float().numpy(),
            scale=np.float32(scale), causal=np.int32(causal),
        )
        print(f"[{name}] written")


REF_FIXTURES = {
    "rope": (("input.bin", "output.bin", "meta.json"), "generate.py:43-79"),
    "swiglu": (("input.bin", "output.bin", "meta.json"), "generate.py:82-101"),
    "fused_add_rmsnorm": (("input_x.bin", "input_residual.bin", "weight.bin", "output_y.bin",
                           "output_h.bin", "meta.json"), "generate.py:104-128"),
}


def copy_reference_fixtures(reference: str):
    for name, (files, where) in REF_FIXTURES.items():
        src = os.path.join(reference, "tests", "fixtures", name)
        dst = os.path.join(HERE, name + "_ref")
        os.makedirs(dst, exist_ok=True)
        digests = {}
        for f in files:
            shutil.copyfile(os.path.join(src, f), os.path.join(dst, f))
            with open(os.path.join(dst, f), "rb") as fh:
                digests[f] = hashlib.sha256(fh.read()).hexdigest()
        with open(os.path.join(dst, "SOURCE.json"), "w") as fh:
            json.dump({"copied_from": f"teenyformers tests/fixtures/{name} ({where})",
                       "sha256": digests}, fh, indent=2)
        print(f"[{name}_ref] copied from {src}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="teenyformers checkout (for rope_ref)")
    args = ap.parse_args()
    if args.reference:
        copy_reference_fixtures(args.reference)
    make_attn()


if __name__ == "__main__":
    main()
