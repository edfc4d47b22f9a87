"""GPU parity of the tensor-parallel Llama decoder layer (one rank) against an
fp32 CPU reference composed from the oracle's pinned pieces
(src/layers/llama_block.rs:55-65)."""
import pytest
import torch

from helpers import assert_bf16_close_scaled, seeded_normal, to_np
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
