"""GPU parity for RoPE and the head transpose/merge, through the C ABI.

Reference behaviour: src/kernels/rope.rs:57-140 (interleaved pairs, theta from
ln(base)), src/kernels/transpose_heads.rs:49-96 (pure copies, bit-exact).
"""
import json
import math
import os

import numpy as np
import pytest
import torch

import oracle
import teenyformers_b200 as tfb
from tests.helpers import F32_ABS, assert_bf16_close, assert_bf16_close_scaled, seeded_normal, to_np

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    yield
    assert tfb.device_status(clear=True) == 0


def test_rope_f32_matches_reference_fixture(cuda_device):
    meta = json.load(open(os.path.join(GOLDEN, "rope_ref", "meta.json")))
    shape = (meta["bh"], meta["s"], meta["head_dim"])
    x = np.fromfile(os.path.join(GOLDEN, "rope_ref", "input.bin"), dtype="<f4").reshape(shape)
    y = np.fromfile(os.path.join(GOLDEN, "rope_ref", "output.bin"), dtype="<f4").reshape(shape)
    op = tfb.RopeOp(meta["head_dim"], meta["rope_base"])
    got = to_np(op.forward(torch.from_numpy(x).to(cuda_device)))
    assert np.abs(got - y).max() < F32_ABS
    back = to_np(op.backward(torch.from_numpy(y).to(cuda_device)))
    assert np.abs(back - x).max() < F32_ABS


@pytest.mark.parametrize("style", [tfb.TF_ROPE_INTERLEAVED, tfb.TF_ROPE_ROTATE_HALF])
@pytest.mark.parametrize("inverse", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rope_vs_oracle(cuda_device, style, inverse, dtype):
    x = seeded_normal((6, 333, 64), seed=11, dtype=dtype, device=cuda_device)
    got = to_np(tfb.rope(x, 10000.0, style, inverse))
    ref = oracle.rope(to_np(x), math.log(10000.0), style, inverse)
    if dtype == torch.float32:
        assert np.abs(got - ref).max() < F32_ABS
    else:
        assert_bf16_close("rope", got, ref)


def test_rope_in_place(cuda_device):
    x = seeded_normal((2, 40, 128), seed=12, dtype=torch.float32, device=cuda_device)
    ref = oracle.rope(to_np(x), math.log(10000.0))
    tfb.rope(x, 10000.0, out=x)
    assert np.abs(to_np(x) - ref).max() < F32_ABS


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(2, 77, 5, 48), (1, 1, 1, 8), (3, 130, 4, 128)])
def test_transpose_merge_bit_exact(cuda_device, dtype, shape):
    B, S, H, D = shape
    x = seeded_normal((B, S, H * D), seed=13, dtype=dtype, device=cuda_device)
    t = tfb.transpose_heads(x, H)
    xb = x.cpu().view(torch.int16 if dtype == torch.bfloat16 else torch.int32).numpy()
    tb = t.cpu().view(torch.int16 if dtype == torch.bfloat16 else torch.int32).numpy()
    assert np.array_equal(tb, oracle.transpose_heads(xb, H))
    m = tfb.merge_heads(t)
    assert torch.equal(m.view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                       x.view(torch.int16 if dtype == torch.bfloat16 else torch.int32))
    # the reference's un-batched [S, D] <-> [H, S, Dh] form
    t2 = tfb.TransposeHeadsOp(H, D).forward(x[0].contiguous())
    assert torch.equal(t2, t[0]) and torch.equal(tfb.MergeHeadsOp(H, D).forward(t2), x[0])


@pytest.mark.parametrize("style", [tfb.TF_ROPE_INTERLEAVED, tfb.TF_ROPE_ROTATE_HALF])
def test_rope_transpose_small_vs_oracle(cuda_device, style):
    x = seeded_normal((2, 95, 6, 128), seed=14, device=cuda_device)
    y = tfb.rope_transpose(x, 500000.0, style)
    ref = oracle.rope_transpose(to_np(x), math.log(500000.0), style)
    assert_bf16_close("rope_transpose", to_np(y), ref)
    dx = tfb.rope_transpose(y, 500000.0, style, inverse=True)
    ref_back = oracle.rope_transpose(to_np(y), math.log(500000.0), style, inverse=True)
    assert_bf16_close("rope_transpose^-1", to_np(dx), ref_back)


@pytest.mark.parametrize("style", [tfb.TF_ROPE_ROTATE_HALF, tfb.TF_ROPE_INTERLEAVED],
                         ids=["rotate_half", "interleaved"])
def test_rope_transpose_config2_full_size(cuda_device, style):
    """BASELINE config #2: x [4, 2048, 32, 128] bf16, theta 1e4; rotate-half (the
    config's wording) and interleaved pairs (the reference's rope.rs)."""
    B, S, H, D = 4, 2048, 32, 128
    x = seeded_normal((B, S, H, D), seed=42, device=cuda_device)
    y = tfb.rope_transpose(x, 10000.0, style)
    ref = oracle.rope_transpose(to_np(x), math.log(10000.0), style)
    assert_bf16_close("config2", to_np(y), ref)
    # the inverse rotation + merge brings x back, to two bf16 roundings (of y and
    # of the result): relative above magnitude 1, where |x| reaches ~5.5 here
    back = tfb.rope_transpose(y, 10000.0, style, inverse=True)
    assert_bf16_close_scaled("config2 inverse", to_np(back), to_np(x))
    # transpose itself is bit-exact at full size
    t = tfb.transpose_heads(x.view(B, S, H * D), H)
    assert torch.equal(t.view(torch.int16), x.permute(0, 2, 1, 3).contiguous().view(torch.int16))
    # size-independent property: position 0 is the identity rotation
    assert torch.equal(y[:, :, 0, :].view(torch.int16), x[:, 0, :, :].view(torch.int16))
