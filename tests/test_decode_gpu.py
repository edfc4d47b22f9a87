"""GPU parity of the KV-cache decode kernel against the oracle: varlen cache
lengths, GQA, several new tokens per sequence (bottom-right causal), key
splits with the combine kernel, and consistency with the causal prefill
kernel when every cached token is new."""
import math

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_bf16_close, seeded_normal, to_np

pytestmark = pytest.mark.gpu


def _reference(q, k, v, lens, scale):
    """Per (sequence, query) oracle call on the visible key prefix."""
    B, Hq, n_q, D = q.shape
    Hkv = k.shape[1]
    o = np.zeros(q.shape, np.float32)
    lse = np.zeros((B, Hq, n_q), np.float32)
    qn, kn, vn = to_np(q), to_np(k), to_np(v)
    for b in range(B):
        for i in range(n_q):
            lim = int(lens[b]) - n_q + i + 1  # visible keys
            ob, lb = oracle.flash_attn2_fwd(qn[b:b + 1, :, i:i + 1], kn[b:b + 1, :, :lim],
                                            vn[b:b + 1, :, :lim], scale, False, n_heads_kv=Hkv)
            o[b, :, i] = ob[0, :, 0]
            lse[b, :, i] = lb[0, :, 0]
    return o, lse


CASES = [  # B, Hq, Hkv, n_q, cap, D, lens (None = random in [n_q, cap])
    (3, 8, 2, 1, 300, 128, [1, 157, 300]),
    (2, 4, 4, 3, 130, 64, [3, 130]),
    (4, 32, 8, 2, 2048, 128, None),
    (1, 8, 1, 1, 8192, 128, [8000]),       # one sequence: split over keys + combine
    (2, 32, 2, 2, 700, 128, [700, 65]),    # G * n_q = 32 rows: two row blocks
    (5, 16, 4, 1, 1000, 64, None),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"b{c[0]}h{c[1]}kv{c[2]}nq{c[3]}cap{c[4]}d{c[5]}")
def test_decode_matches_oracle(cuda_device, case):
    import teenyformers_b200 as tfb
    B, Hq, Hkv, n_q, cap, D, lens = case
    if lens is None:
        rng = np.random.default_rng(B * 1000 + cap)
        lens = rng.integers(n_q, cap + 1, size=B).tolist()
    q = seeded_normal((B, Hq, n_q, D), 21, device=cuda_device)
    k = seeded_normal((B, Hkv, cap, D), 22, device=cuda_device)
    v = seeded_normal((B, Hkv, cap, D), 23, device=cuda_device)
    seq = torch.tensor(lens, dtype=torch.int32, device=cuda_device)
    scale = 1.0 / math.sqrt(D)
    o, lse = tfb.flash_attn2_decode(q, k, v, seq, scale)
    torch.cuda.synchronize()
    ro, rl = _reference(q, k, v, lens, scale)
    assert_bf16_close("o", to_np(o), ro)
    assert np.abs(to_np(lse) - rl).max() < 2e-3


def test_decode_equals_causal_prefill_when_all_tokens_are_new(cuda_device):
    import teenyformers_b200 as tfb
    B, H, S, D = 2, 4, 192, 128
    q = seeded_normal((B, H, S, D), 31, device=cuda_device)
    k = seeded_normal((B, H, S, D), 32, device=cuda_device)
    v = seeded_normal((B, H, S, D), 33, device=cuda_device)
    seq = torch.full((B,), S, dtype=torch.int32, device=cuda_device)
    o_dec, l_dec = tfb.flash_attn2_decode(q, k, v, seq, D ** -0.5)
    o_pre, l_pre = tfb.flash_attn2_fwd(q, k, v, D ** -0.5, True)
    assert_bf16_close("o", to_np(o_dec), to_np(o_pre))
    assert float((l_dec - l_pre).abs().max()) < 2e-3


def test_decode_rejects_bad_arguments(cuda_device):
    import teenyformers_b200 as tfb
    q = torch.zeros((1, 6, 1, 128), dtype=torch.bfloat16, device=cuda_device)
    k = torch.zeros((1, 4, 64, 128), dtype=torch.bfloat16, device=cuda_device)
    seq = torch.ones(1, dtype=torch.int32, device=cuda_device)
    with pytest.raises(tfb.TfError):  # 6 query heads over 4 KV heads
        tfb.flash_attn2_decode(q, k, k, seq, 0.1)
