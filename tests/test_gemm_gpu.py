"""GPU parity of the tcgen05 GEMM and its fused epilogues, through the C ABI:

  linear            the Llama block's Linear (teeny-core; src/layers/mod.rs:54-65)
  heads-layout A    o_proj reading the attention output with MergeHeads folded in
                    (transpose_heads.rs:86-95)
  linear_swiglu     gate/up projection + SwiGLU (ffn.rs:47-56, swiglu.rs:56-95)
  linear_qkv_rope   Q/K/V projections + TransposeHeads + RoPE (attention.rs:89-123,
                    rope.rs:57-96), both pair styles, with and without rotation
  linear_push       the tensor-parallel reduce-scatter placement (rank o's rows to
                    rank o's receive buffer, slot [rank]); two "ranks" emulated on
                    one GPU by giving both receive buffers in local memory

Each is compared with a plain PyTorch fp32 GEMM on the same bf16 inputs
(TF32 off), followed by the oracle's restatement of the fused op.
"""
import math

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_bf16_close_scaled, seeded_normal, to_np

pytestmark = pytest.mark.gpu


def _w(shape, seed, dev):
    k = shape[-1]
    return (seeded_normal(shape, seed, dtype=torch.float32) / math.sqrt(k)).to(
        torch.bfloat16).to(dev)


def _mm32(x, w):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return torch.matmul(x.float(), w.float().t())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 256), (300, 136, 72),
                                   (1000, 1032, 520), (2048, 768, 4096), (130, 8, 8),
                                   (4096, 4096, 1024)])
def test_linear_matches_fp32(cuda_device, m, n, k):
    import teenyformers_b200 as tfb
    x = seeded_normal((m, k), 11).to(cuda_device)
    w = _w((n, k), 12, cuda_device)
    y = tfb.linear(x, w)
    ref = _mm32(x, w)
    assert_bf16_close_scaled("linear", to_np(y), to_np(ref), tol=1e-2, rl2=4e-3)
    # every output written (no stale tile): compare against cuBLAS's bf16 GEMM too
    cub = torch.matmul(x, w.t())
    assert float((y.float() - cub.float()).abs().max()) <= 2e-2 * max(1.0, float(cub.abs().max()))
    assert tfb.device_status() == 0


def test_linear_is_deterministic(cuda_device):
    import teenyformers_b200 as tfb
    x = seeded_normal((1024, 512), 21).to(cuda_device)
    w = _w((768, 512), 22, cuda_device)
    a = tfb.linear(x, w)
    b = tfb.linear(x, w)
    assert torch.equal(a, b)


@pytest.mark.parametrize("B,H,S,n", [(2, 4, 256, 512), (1, 32, 128, 256), (3, 2, 384, 136)])
def test_linear_heads_layout_folds_merge(cuda_device, B, H, S, n):
    import teenyformers_b200 as tfb
    o = seeded_normal((B, H, S, 128), 31).to(cuda_device)
    w = _w((n, H * 128), 32, cuda_device)
    y = tfb.linear(o, w, heads_seq=S)
    merged = tfb.merge_heads(o)                       # [B, S, H*128]
    y2 = tfb.linear(merged, w)
    assert y.shape == (B, S, n)
    assert torch.equal(y, y2), "heads-layout A must equal merge_heads + linear bit for bit"
    assert_bf16_close_scaled("heads", to_np(y), to_np(_mm32(merged, w)), tol=1e-2, rl2=4e-3)


@pytest.mark.parametrize("m,d_ff,k", [(128, 128, 64), (300, 256, 136), (2048, 1792, 512),
                                      (4096, 3584, 4096)])
def test_linear_swiglu_matches_oracle(cuda_device, m, d_ff, k):
    import teenyformers_b200 as tfb
    x = seeded_normal((m, k), 41).to(cuda_device)
    wg = _w((d_ff, k), 42, cuda_device)
    wu = _w((d_ff, k), 43, cuda_device)
    blocks = tfb.swiglu_weight_blocks(wg, wu)
    y = tfb.linear_swiglu(x, blocks)
    z = torch.cat([_mm32(x, wg), _mm32(x, wu)], dim=-1)
    ref = oracle.swiglu(to_np(z))
    assert_bf16_close_scaled("swiglu", to_np(y), ref, tol=1e-2, rl2=4e-3)


@pytest.mark.parametrize("B,S,Hq,Hkv,d,style,base", [
    (2, 256, 4, 2, 256, 0, 1e4),
    (1, 128, 2, 1, 512, 1, 5e5),
    (1, 384, 1, 1, 128, 0, 5e5),     # 3 heads: the last tile holds one head
    (2, 128, 8, 2, 1024, 1, 1e4),
])
@pytest.mark.parametrize("rotate", [True, False])
def test_linear_qkv_rope_matches_oracle(cuda_device, B, S, Hq, Hkv, d, style, base, rotate):
    import teenyformers_b200 as tfb
    x = seeded_normal((B, S, d), 51).to(cuda_device)
    wq = _w((Hq * 128, d), 52, cuda_device)
    wk = _w((Hkv * 128, d), 53, cuda_device)
    wv = _w((Hkv * 128, d), 54, cuda_device)
    w_qkv = torch.cat([wq, wk, wv]).contiguous()
    table = tfb.rope_table(S, 128, base, cuda_device) if rotate else None
    q, k, v = tfb.linear_qkv_rope(x, w_qkv, Hq, Hkv, table, style)
    lnb = math.log(base)
    for name, got, w_, H in (("q", q, wq, Hq), ("k", k, wk, Hkv)):
        proj = to_np(_mm32(x, w_)).reshape(B, S, H, 128)
        ref = (oracle.rope_transpose(proj, lnb, style) if rotate
               else np.ascontiguousarray(proj.transpose(0, 2, 1, 3)))
        assert_bf16_close_scaled(name, to_np(got), ref, tol=1e-2, rl2=4e-3)
    refv = to_np(_mm32(x, wv)).reshape(B, S, Hkv, 128).transpose(0, 2, 1, 3)
    assert_bf16_close_scaled("v", to_np(v), np.ascontiguousarray(refv), tol=1e-2, rl2=4e-3)


def test_rope_table_matches_rope_kernel_angles(cuda_device):
    """The table's rotation equals the standalone RoPE kernel's on a unit input."""
    import teenyformers_b200 as tfb
    S, D, base = 256, 128, 5e5
    t = tfb.rope_table(S, D, base, cuda_device).cpu().numpy()       # [S, 64, 2]
    ones = torch.zeros((1, S, D), dtype=torch.float32)
    ones[..., 0::2] = 1.0                                              # (1, 0) pairs
    rot = tfb.rope(ones.to(cuda_device), base).cpu().numpy()[0]       # interleaved
    np.testing.assert_array_equal(rot[:, 0::2], t[:, :, 0])
    np.testing.assert_array_equal(rot[:, 1::2], t[:, :, 1])


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("heads", [False, True])
def test_linear_push_places_rows_by_owner(cuda_device, heads, world):
    """`world` emulated ranks push their partial products; receive buffer o then holds
    rank r's rows [o*slice, (o+1)*slice) at slot r, bit-equal to the plain GEMM."""
    import teenyformers_b200 as tfb
    B, S, H, n = 2, 128 * world, 4, 512
    m, k = B * S, H * 128
    slice_rows = m // world
    recv = [torch.full((world, slice_rows, n), float("nan"), dtype=torch.bfloat16,
                       device=cuda_device) for _ in range(world)]
    ptrs = [r.data_ptr() for r in recv]
    w = _w((n, k), 61, cuda_device)
    partial = []
    for rank in range(world):
        if heads:
            a = seeded_normal((B, H, S, 128), 62 + rank).to(cuda_device)
            tfb.linear_push(a, w, ptrs, rank, world, heads_seq=S)
            partial.append(tfb.linear(a, w, heads_seq=S).reshape(m, n))
        else:
            a = seeded_normal((m, k), 62 + rank).to(cuda_device)
            tfb.linear_push(a, w, ptrs, rank, world)
            partial.append(tfb.linear(a, w))
    torch.cuda.synchronize()
    for o in range(world):
        for r in range(world):
            assert torch.equal(recv[o][r], partial[r][o * slice_rows:(o + 1) * slice_rows]), (o, r)
    assert tfb.device_status() == 0
