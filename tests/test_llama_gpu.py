"""GPU parity of the tensor-parallel Llama decoder layer (one rank) against an
fp32 CPU reference composed from the oracle's pinned pieces
(src/layers/llama_block.rs:55-65)."""
import pytest
import torch

from helpers import assert_bf16_close_scaled, rel_l2, seeded_normal, to_np
from llama_ref import layer_ref_fp32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,S,d,H,Hkv,D,d_ff", [
    (1, 128, 256, 4, 2, 64, 512),      # GQA 2:1
    (2, 77, 512, 4, 4, 128, 1024),     # MHA, ragged sequence
    (1, 256, 1024, 8, 2, 128, 2816),   # Llama-shaped ratios
    (2, 256, 512, 4, 1, 128, 1536),    # GQA 4:1, two sequences
])
@pytest.mark.parametrize("fused", [True, False])
def test_llama_layer_matches_fp32_reference(cuda_device, B, S, d, H, Hkv, D, d_ff, fused):
    from teenyformers_b200.llama import LlamaLayerConfig, LlamaLayerTP, init_full_weights
    cfg = LlamaLayerConfig(d_model=d, n_heads=H, n_kv_heads=Hkv, head_dim=D, d_ff=d_ff)
    w = init_full_weights(cfg, seed=7, device=cuda_device)
    x = seeded_normal((B, S, d), 11).to(cuda_device)
    layer = LlamaLayerTP(cfg, w, fused=fused)
    assert layer.fused_ok(B, S) == (fused and D == 128 and S % 128 == 0)
    y = layer.forward(x)
    torch.cuda.synchronize()
    ref = layer_ref_fp32(x.float().cpu(), w, cfg, H, Hkv)
    # bf16 activations between the kernels and GEMMs: the layer output is a
    # residual sum of magnitude > 1, checked with the scaled bf16 bound
    assert_bf16_close_scaled("layer", to_np(y), ref.numpy(), tol=3e-2)


@pytest.mark.parametrize("D,S", [(64, 64), (128, 128)])
def test_llama_layer_rotate_half_style(cuda_device, D, S):
    from teenyformers_b200 import TF_ROPE_ROTATE_HALF
    from teenyformers_b200.llama import LlamaLayerConfig, LlamaLayerTP, init_full_weights
    cfg = LlamaLayerConfig(d_model=256, n_heads=4, n_kv_heads=1, head_dim=D, d_ff=512,
                           rope_style=TF_ROPE_ROTATE_HALF)
    w = init_full_weights(cfg, seed=3, device=cuda_device)
    x = seeded_normal((1, S, 256), 5).to(cuda_device)
    y = LlamaLayerTP(cfg, w).forward(x)
    ref = layer_ref_fp32(x.float().cpu(), w, cfg, 4, 1)
    assert_bf16_close_scaled("layer", to_np(y), ref.numpy(), tol=3e-2)


@pytest.mark.parametrize("B,S,d,H,Hkv,D,d_ff", [
    (1, 128, 256, 4, 2, 128, 512),   # fused layers
    (2, 77, 256, 4, 4, 64, 512),     # separate-kernel layers (head_dim 64, ragged S)
])
def test_llama_model_stack_matches_reference(cuda_device, B, S, d, H, Hkv, D, d_ff):
    """Two layers + the final RMSNorm (src/llama.rs:65-81) against the fp32
    composition of the oracle layer."""
    from llama_ref import model_ref_fp32
    from teenyformers_b200.llama import LlamaLayerConfig, LlamaModelTP, init_model_weights
    cfg = LlamaLayerConfig(d_model=d, n_heads=H, n_kv_heads=Hkv, head_dim=D, d_ff=d_ff)
    layers, norm = init_model_weights(cfg, 2, seed=21, device=cuda_device)
    x = seeded_normal((B, S, d), 12).to(cuda_device)
    model = LlamaModelTP(cfg, layers, norm)
    y = model.forward(x)
    torch.cuda.synchronize()
    ref = model_ref_fp32(x.float().cpu(), layers, norm, cfg, H, Hkv)
    assert_bf16_close_scaled("stack", to_np(y), ref.numpy(), tol=3e-2)


def test_llama_layer_cublas_arm_matches_reference(cuda_device):
    """The explicitly named cuBLAS comparison arm computes the same layer."""
    from teenyformers_b200.llama import LlamaLayerConfig, LlamaLayerTP, init_full_weights
    cfg = LlamaLayerConfig(d_model=256, n_heads=4, n_kv_heads=2, head_dim=128, d_ff=512)
    w = init_full_weights(cfg, seed=8, device=cuda_device)
    x = seeded_normal((1, 128, 256), 13).to(cuda_device)
    y = LlamaLayerTP(cfg, w, fused=False, projections="cublas").forward(x)
    ref = layer_ref_fp32(x.float().cpu(), w, cfg, 4, 2)
    assert_bf16_close_scaled("cublas arm", to_np(y), ref.numpy(), tol=3e-2)


@pytest.mark.parametrize("B,St,Se,d,H,Hkv,D,d_ff", [
    (2, 96, 160, 256, 4, 2, 64, 512),     # cross-attention Sq < Sk, GQA 2:1
    (1, 128, 200, 512, 4, 4, 128, 1024),  # fused QKV self-attention, ragged encoder
    (1, 256, 72, 256, 2, 1, 128, 320),    # Sq > Sk, d_ff not a multiple of 128
])
def test_decoder_block_matches_reference(cuda_device, B, St, Se, d, H, Hkv, D, d_ff):
    """DecoderBlock (src/layers/decoder_block.rs:68-81): causal self-attention,
    non-causal cross-attention over the encoder output (Sq != Sk), SwiGLU FFN."""
    from llama_ref import decoder_block_ref_fp32
    from teenyformers_b200.decoder import DecoderBlockTP, init_decoder_block_weights
    from teenyformers_b200.llama import LlamaLayerConfig
    cfg = LlamaLayerConfig(d_model=d, n_heads=H, n_kv_heads=Hkv, head_dim=D, d_ff=d_ff,
                           rope_base=10000.0)
    w = init_decoder_block_weights(cfg, seed=31, device=cuda_device)
    tgt = seeded_normal((B, St, d), 14).to(cuda_device)
    enc = seeded_normal((B, Se, d), 15).to(cuda_device)
    y = DecoderBlockTP(cfg, w).forward(tgt, enc)
    torch.cuda.synchronize()
    ref = decoder_block_ref_fp32(tgt.float().cpu(), enc.float().cpu(), w, cfg, H, Hkv)
    assert_bf16_close_scaled("decoder block", to_np(y), ref.numpy(), tol=3e-2)


def test_decoder_stack_matches_reference(cuda_device):
    """Two decoder blocks + the final RMSNorm (src/decoder.rs:48-53)."""
    from llama_ref import decoder_ref_fp32
    from teenyformers_b200.decoder import DecoderTP, init_decoder_block_weights
    from teenyformers_b200.llama import LlamaLayerConfig
    cfg = LlamaLayerConfig(d_model=256, n_heads=2, n_kv_heads=2, head_dim=128, d_ff=512,
                           rope_base=10000.0)
    blocks = [init_decoder_block_weights(cfg, seed=40 + i, device=cuda_device) for i in range(2)]
    norm = init_decoder_block_weights(cfg, seed=42, device=cuda_device)["norm1"]
    tgt = seeded_normal((1, 128, 256), 16).to(cuda_device)
    enc = seeded_normal((1, 96, 256), 17).to(cuda_device)
    y = DecoderTP(cfg, blocks, norm).forward(tgt, enc)
    ref = decoder_ref_fp32(tgt.float().cpu(), enc.float().cpu(), blocks, norm, cfg, 2, 2)
    assert_bf16_close_scaled("decoder", to_np(y), ref.numpy(), tol=3e-2)


def test_config5_layer_full_size_sampled_rows(cuda_device):
    """BASELINE config #5's layer (d=4096, 32 query / 8 KV heads, head_dim 128,
    SwiGLU 14336, eps 1e-5, theta 5e5, weights N(0, 0.02)) at S=4096, one
    sequence, on the fused path: the first and the last 64 token rows.

    Against the all-fp32 layer: rel-L2 <= 1e-2.  Against
    the fp32 layer with the fused path's bf16 storage points, elementwise: the
    attention's allowed error (bf16 P, max-abs 2e-2 on O) passes through
    o_proj, gate/up and down GEMMs of fan-in 4096-14336, so the largest of
    262,144 differences lands near 5e-2: the elementwise bar is max-abs
    (scaled by max(1, |ref|)) <= 8e-2, with rel-L2 <= 1e-2 against both."""
    from llama_ref import layer_rows_ref_fp32
    from teenyformers_b200.llama import LlamaLayerConfig, LlamaLayerTP, init_full_weights
    cfg = LlamaLayerConfig()  # the Llama-3-8B shape of config #5
    assert (cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.d_ff) == (4096, 32, 8, 14336)
    B, S = 1, 4096
    w = init_full_weights(cfg, seed=5, device=cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(55)
    x = torch.randn((B, S, cfg.d_model), generator=g, device=cuda_device, dtype=torch.bfloat16)
    layer = LlamaLayerTP(cfg, w)
    assert layer.fused_ok(B, S)
    y = layer.forward(x)
    torch.cuda.synchronize()
    xc = x.float().cpu()
    for lo, hi in ((0, 64), (S - 64, S)):
        got = to_np(y[:, lo:hi])
        ref = layer_rows_ref_fp32(xc, w, cfg, cfg.n_heads, cfg.n_kv_heads, lo, hi).numpy()
        assert rel_l2(got, ref) <= 1e-2, f"rows {lo}:{hi} rel-L2 {rel_l2(got, ref):.3e}"
        ref_b = layer_rows_ref_fp32(xc, w, cfg, cfg.n_heads, cfg.n_kv_heads, lo, hi,
                                    bf16_points=True).numpy()
        assert_bf16_close_scaled(f"rows {lo}:{hi} (bf16 storage points)", got, ref_b, tol=8e-2)
