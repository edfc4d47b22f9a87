"""Pins the CPU oracle (oracle/oracle.c) before it is trusted as the checker.

- RoPE: against the reference's own golden vector (teenyformers
  tests/fixtures/rope, checked there at abs-tol 1e-4 by
  tests/kernel_execution.rs:169-215), copied to tests/golden/rope_ref.
- Attention fwd/bwd: against float64 torch known-answer vectors with the
  reference kernel's semantics (tests/golden/make_golden.py).  The reference's
  attention kernels cannot be run here, so this is a second witness.
- Transpose / merge: bit-exact against numpy.
"""
import glob
import hashlib
import json
import math
import os

import numpy as np
import pytest

import oracle
from tests.helpers import F32_ABS

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_rope_fixture_integrity():
    meta = json.load(open(os.path.join(GOLDEN, "rope_ref", "SOURCE.json")))
    for f, digest in meta["sha256"].items():
        with open(os.path.join(GOLDEN, "rope_ref", f), "rb") as fh:
            assert hashlib.sha256(fh.read()).hexdigest() == digest, f


def _rope_fixture():
    meta = json.load(open(os.path.join(GOLDEN, "rope_ref", "meta.json")))
    shape = (meta["bh"], meta["s"], meta["head_dim"])
    x = np.fromfile(os.path.join(GOLDEN, "rope_ref", "input.bin"), dtype="<f4").reshape(shape)
    y = np.fromfile(os.path.join(GOLDEN, "rope_ref", "output.bin"), dtype="<f4").reshape(shape)
    return x, y, meta["rope_base"]


def test_oracle_rope_matches_reference_fixture():
    x, y, base = _rope_fixture()
    got = oracle.rope(x, math.log(base), oracle.ROPE_INTERLEAVED)
    assert np.abs(got - y).max() < F32_ABS


def test_oracle_rope_is_interleaved_not_rotate_half():
    x, y, base = _rope_fixture()
    got = oracle.rope(x, math.log(base), oracle.ROPE_ROTATE_HALF)
    assert np.abs(got - y).max() > 0.1


@pytest.mark.parametrize("style", [oracle.ROPE_INTERLEAVED, oracle.ROPE_ROTATE_HALF])
def test_oracle_rope_inverse_roundtrip(style):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 50, 64)).astype(np.float32)
    y = oracle.rope(x, math.log(10000.0), style)
    back = oracle.rope(y, math.log(10000.0), style, inverse=True)
    assert np.abs(back - x).max() < 1e-5


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "attn_*.npz"))),
                         ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_attention_matches_fp64_witness(path):
    z = np.load(path)
    scale, causal = float(z["scale"]), bool(z["causal"])
    o, lse = oracle.flash_attn2_fwd(z["q"], z["k"], z["v"], scale, causal)
    assert np.abs(o - z["o"]).max() < F32_ABS
    assert np.abs(lse - z["lse"]).max() < F32_ABS
    dq, dk, dv = oracle.flash_attn2_bwd(z["q"], z["k"], z["v"], z["o"], z["do"], z["lse"],
                                        scale, causal)
    for name, got in (("dq", dq), ("dk", dk), ("dv", dv)):
        assert np.abs(got - z[name]).max() < F32_ABS, name


def test_oracle_fwd_row_sample_matches_full():
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 2, 40, 32)).astype(np.float32)
    k = rng.standard_normal((1, 2, 40, 32)).astype(np.float32)
    v = rng.standard_normal((1, 2, 40, 32)).astype(np.float32)
    o, lse = oracle.flash_attn2_fwd(q, k, v, 0.2, True)
    o2, lse2 = oracle.flash_attn2_fwd(q, k, v, 0.2, True, bh_range=(1, 2), q_range=(7, 19))
    assert np.array_equal(o2[0, 1, 7:19], o[0, 1, 7:19])
    assert np.isnan(o2[0, 0]).all()


@pytest.mark.parametrize("dtype", [np.float32, np.uint16])
def test_oracle_transpose_merge_bit_exact(dtype):
    rng = np.random.default_rng(2)
    B, S, H, D = 2, 5, 3, 16
    x = rng.integers(0, 2**16, size=(B, S, H * D)).astype(dtype)
    t = oracle.transpose_heads(x, H)
    assert np.array_equal(t, x.reshape(B, S, H, D).transpose(0, 2, 1, 3))
    m = oracle.merge_heads(t)
    assert np.array_equal(m.reshape(B, S, H * D), x)


def test_oracle_rope_transpose_composes():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 9, 4, 32)).astype(np.float32)
    y = oracle.rope_transpose(x, math.log(500000.0), oracle.ROPE_ROTATE_HALF)
    ref = oracle.rope(np.ascontiguousarray(x.transpose(0, 2, 1, 3)), math.log(500000.0),
                      oracle.ROPE_ROTATE_HALF)
    assert np.array_equal(y, ref)
    back = oracle.rope_transpose(y, math.log(500000.0), oracle.ROPE_ROTATE_HALF, inverse=True)
    assert np.abs(back - x).max() < 1e-5


def test_oracle_swiglu_matches_reference_fixture():
    meta = json.load(open(os.path.join(GOLDEN, "swiglu_ref", "meta.json")))
    m, d_ff = meta["m"], meta["d_ff"]
    z = np.fromfile(os.path.join(GOLDEN, "swiglu_ref", "input.bin"), dtype="<f4").reshape(m, 2 * d_ff)
    out = np.fromfile(os.path.join(GOLDEN, "swiglu_ref", "output.bin"), dtype="<f4").reshape(m, d_ff)
    assert np.abs(oracle.swiglu(z) - out).max() < F32_ABS


def test_oracle_fused_add_rmsnorm_matches_reference_fixture():
    d = os.path.join(GOLDEN, "fused_add_rmsnorm_ref")
    meta = json.load(open(os.path.join(d, "meta.json")))
    m, n = meta["m"], meta["n"]
    rd = lambda f, shape: np.fromfile(os.path.join(d, f), dtype="<f4").reshape(shape)
    y, h = oracle.rmsnorm(rd("input_x.bin", (m, n)), rd("weight.bin", (n,)), meta["eps"],
                          residual=rd("input_residual.bin", (m, n)))
    assert np.abs(y - rd("output_y.bin", (m, n))).max() < F32_ABS
    assert np.abs(h - rd("output_h.bin", (m, n))).max() < F32_ABS


def test_reference_fixture_integrity_all():
    for name in ("swiglu_ref", "fused_add_rmsnorm_ref"):
        meta = json.load(open(os.path.join(GOLDEN, name, "SOURCE.json")))
        for f, digest in meta["sha256"].items():
            with open(os.path.join(GOLDEN, name, f), "rb") as fh:
                assert hashlib.sha256(fh.read()).hexdigest() == digest, (name, f)
