"""Host-side routing of the Llama layer, stack and decoder block (no GPU): with
the library's ops replaced by shape-only fakes and torch.matmul made to raise,
every default path (fused, and the separate-kernel path that shapes outside
the fused epilogues take) must reach only this library's entry points.  The
cuBLAS projections exist only behind the explicit ``projections="cublas"``."""
import pytest
import torch

import teenyformers_b200.ops as ops
from teenyformers_b200.decoder import DecoderBlockTP, init_decoder_block_weights
from teenyformers_b200.llama import (LlamaLayerConfig, LlamaLayerTP, LlamaModelTP,
                                     init_full_weights, init_model_weights)


@pytest.fixture
def fake_ops(monkeypatch):
    calls = []

    def rec(name, fn):
        def f(*a, **k):
            calls.append(name)
            return fn(*a, **k)
        monkeypatch.setattr(ops, name, f)

    def linear(x, w, out=None, heads_seq=0, residual=None):
        # the GEMM's host check: heads-layout A needs 128-row blocks per head
        assert heads_seq % 128 == 0 and x.shape[-1] == 128 if heads_seq else True
        lead = (x.shape[0], heads_seq) if heads_seq else tuple(x.shape[:-1])
        return torch.zeros(lead + (w.shape[0],), dtype=x.dtype)

    rec("rmsnorm", lambda x, w, eps, residual=None, out=None, residual_out=None:
        (torch.zeros_like(x), torch.zeros_like(x)) if residual is not None else torch.zeros_like(x))
    rec("linear", linear)
    rec("linear_swiglu", lambda x, wb, out=None:
        torch.zeros(tuple(x.shape[:-1]) + (wb.shape[0] // 2,), dtype=x.dtype))
    rec("swiglu", lambda z, out=None: torch.zeros(tuple(z.shape[:-1]) + (z.shape[-1] // 2,),
                                                  dtype=z.dtype))
    rec("swiglu_weight_blocks", lambda g, u: torch.cat([g, u]))
    rec("rope_table", lambda S, D, base, dev: torch.zeros(S, D // 2, 2))
    rec("linear_qkv_rope", lambda x, w, hq, hkv, table, style=0, outs=None: (
        torch.zeros(x.shape[0], hq, x.shape[1], 128, dtype=x.dtype),
        torch.zeros(x.shape[0], hkv, x.shape[1], 128, dtype=x.dtype),
        torch.zeros(x.shape[0], hkv, x.shape[1], 128, dtype=x.dtype)))
    rec("rope_transpose", lambda x, base, style=0, inverse=False, out=None:
        torch.zeros(x.shape[0], x.shape[2], x.shape[1], x.shape[3], dtype=x.dtype))
    rec("transpose_heads", lambda x, h: torch.zeros(x.shape[0], h, x.shape[1], x.shape[2] // h,
                                                    dtype=x.dtype))
    rec("merge_heads", lambda o: torch.zeros(o.shape[0], o.shape[2], o.shape[1] * o.shape[3],
                                             dtype=o.dtype))
    def attn(q, k, v, scale, causal, out=None, lse=None):
        calls.append(("causal" if causal else "non-causal", q.shape[2], k.shape[2]))
        return torch.zeros_like(q), torch.zeros(q.shape[:-1])
    rec("flash_attn2_fwd", attn)

    def no_matmul(*a, **k):
        raise AssertionError("torch.matmul reached on a default path")
    monkeypatch.setattr(torch, "matmul", no_matmul)
    return calls


@pytest.mark.parametrize("D,S,fused", [(128, 128, True), (128, 77, True), (64, 128, True),
                                       (128, 128, False)])
def test_layer_default_paths_use_only_library_kernels(fake_ops, D, S, fused):
    cfg = LlamaLayerConfig(d_model=256, n_heads=256 // D, n_kv_heads=1, head_dim=D, d_ff=256)
    w = init_full_weights(cfg, seed=0, device="cpu")
    layer = LlamaLayerTP(cfg, w, fused=fused)
    y = layer.forward(torch.zeros(2, S, 256, dtype=torch.bfloat16))
    assert y.shape == (2, S, 256)
    assert ("linear_qkv_rope" in fake_ops) == (fused and D == 128 and S % 128 == 0)
    assert "flash_attn2_fwd" in fake_ops


def test_stack_and_decoder_block_use_only_library_kernels(fake_ops):
    cfg = LlamaLayerConfig(d_model=256, n_heads=2, n_kv_heads=1, head_dim=128, d_ff=256)
    layers, norm = init_model_weights(cfg, 2, seed=0, device="cpu")
    y = LlamaModelTP(cfg, layers, norm).forward(torch.zeros(1, 128, 256, dtype=torch.bfloat16))
    assert y.shape == (1, 128, 256)
    w = init_decoder_block_weights(cfg, seed=1, device="cpu")
    out = DecoderBlockTP(cfg, w).forward(torch.zeros(1, 96, 256, dtype=torch.bfloat16),
                                         torch.zeros(1, 160, 256, dtype=torch.bfloat16))
    assert out.shape == (1, 96, 256)
    attn = [c for c in fake_ops if isinstance(c, tuple)]
    # two causal layers of the stack, then the block's causal self-attention and
    # its non-causal cross-attention with Sq = 96 queries against Sk = 160 keys
    assert attn == [("causal", 128, 128)] * 2 + [("causal", 96, 96), ("non-causal", 96, 160)]


def test_cublas_arm_is_explicit_only():
    cfg = LlamaLayerConfig(d_model=256, n_heads=2, n_kv_heads=1, head_dim=128, d_ff=256)
    w = init_full_weights(cfg, seed=0, device="cpu")
    with pytest.raises(ValueError):
        LlamaLayerTP(cfg, w, projections="cublas")  # needs fused=False
    with pytest.raises(ValueError):
        LlamaLayerTP(cfg, w, fused=False, projections="torch")
    assert LlamaLayerTP(cfg, w, fused=False, projections="cublas").projections == "cublas"


def test_layer_rows_reference_equals_full_reference():
    """The sampled-rows fp32 layer used by the full-size config #5 check
    equals the full fp32 layer on those rows (CPU, oracle pieces)."""
    import os
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    from llama_ref import layer_ref_fp32, layer_rows_ref_fp32
    cfg = LlamaLayerConfig(d_model=128, n_heads=4, n_kv_heads=2, head_dim=32, d_ff=256)
    w = init_full_weights(cfg, seed=3, device="cpu", dtype=torch.float32)
    x = torch.randn(2, 80, 128, generator=torch.Generator().manual_seed(4))
    full = layer_ref_fp32(x, w, cfg, 4, 2)
    for lo, hi in ((0, 16), (50, 80)):
        rows = layer_rows_ref_fp32(x, w, cfg, 4, 2, lo, hi)
        assert float((rows - full[:, lo:hi]).abs().max()) < 1e-4
