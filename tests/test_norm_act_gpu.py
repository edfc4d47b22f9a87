"""GPU parity of the Llama block's RMSNorm (fused residual add) and SwiGLU
kernels through the C ABI, against the oracle on the same bf16 inputs and
against the reference's own fixtures (fused_add_rmsnorm.rs:53-110,
swiglu.rs:56-95)."""
import json
import os

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_bf16_close_scaled, seeded_normal, to_np

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")

pytestmark = pytest.mark.gpu


def _bf16(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(torch.bfloat16)


@pytest.mark.parametrize("rows,cols", [(1, 8), (3, 64), (17, 1000), (64, 4096), (5, 8192),
                                       (1000, 2048)])
@pytest.mark.parametrize("fused", [False, True])
def test_rmsnorm_matches_oracle(cuda_device, rows, cols, fused):
    import teenyformers_b200 as tfb
    x = seeded_normal((rows, cols), 1).to(cuda_device).to(torch.bfloat16)
    r = seeded_normal((rows, cols), 2).to(cuda_device).to(torch.bfloat16) if fused else None
    w = (1.0 + 0.1 * seeded_normal((cols,), 3)).to(cuda_device).to(torch.bfloat16)
    got = tfb.rmsnorm(x, w, 1e-5, residual=r)
    ref_y, ref_h = oracle.rmsnorm(to_np(x), to_np(w), 1e-5, residual=None if r is None else to_np(r))
    if fused:
        y, h = got
        assert_bf16_close_scaled("h", to_np(h), ref_h)
    else:
        y = got
    assert_bf16_close_scaled("y", to_np(y), ref_y)


def test_rmsnorm_reference_fixture(cuda_device):
    import teenyformers_b200 as tfb
    d = os.path.join(GOLDEN, "fused_add_rmsnorm_ref")
    meta = json.load(open(os.path.join(d, "meta.json")))
    m, n = meta["m"], meta["n"]
    rd = lambda f, shape: np.fromfile(os.path.join(d, f), dtype="<f4").reshape(shape)
    y, h = tfb.rmsnorm(_bf16(rd("input_x.bin", (m, n)), cuda_device),
                       _bf16(rd("weight.bin", (n,)), cuda_device), meta["eps"],
                       residual=_bf16(rd("input_residual.bin", (m, n)), cuda_device))
    # fixture computed in fp32 from unrounded inputs: bf16 input + output rounding
    # (2^-9 each, relative) stay inside the scaled bound
    assert_bf16_close_scaled("y", to_np(y), rd("output_y.bin", (m, n)))
    assert_bf16_close_scaled("h", to_np(h), rd("output_h.bin", (m, n)))


def test_rmsnorm_rejects_bad_shapes(cuda_device):
    import teenyformers_b200 as tfb
    x = torch.zeros((4, 12), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(tfb.TfError):
        tfb.rmsnorm(x, torch.ones(12, dtype=torch.bfloat16, device=cuda_device), 1e-5)
    x = torch.zeros((2, 8200), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(tfb.TfError):
        tfb.rmsnorm(x, torch.ones(8200, dtype=torch.bfloat16, device=cuda_device), 1e-5)


@pytest.mark.parametrize("rows,d_ff", [(1, 8), (7, 96), (128, 14336), (1031, 512)])
def test_swiglu_matches_oracle(cuda_device, rows, d_ff):
    import teenyformers_b200 as tfb
    z = (2.0 * seeded_normal((rows, 2 * d_ff), 4)).to(cuda_device).to(torch.bfloat16)
    y = tfb.swiglu(z)
    assert_bf16_close_scaled("swiglu", to_np(y), oracle.swiglu(to_np(z)))


def test_swiglu_reference_fixture(cuda_device):
    import teenyformers_b200 as tfb
    d = os.path.join(GOLDEN, "swiglu_ref")
    meta = json.load(open(os.path.join(d, "meta.json")))
    m, d_ff = meta["m"], meta["d_ff"]
    z = np.fromfile(os.path.join(d, "input.bin"), dtype="<f4").reshape(m, 2 * d_ff)
    out = np.fromfile(os.path.join(d, "output.bin"), dtype="<f4").reshape(m, d_ff)
    y = tfb.swiglu(_bf16(z, cuda_device))
    assert_bf16_close_scaled("swiglu", to_np(y), out)
