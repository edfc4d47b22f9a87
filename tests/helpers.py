"""Shared tolerance checks and seeded inputs for the parity tests."""
from __future__ import annotations

import numpy as np
import torch

# north_star parity bar for bf16 attention / RoPE / gradients vs the fp32 oracle
BF16_MAX_ABS = 2e-2
BF16_REL_L2 = 1e-2
# the reference's own test tolerance (tests/kernel_execution.rs:36), fp32 paths
F32_ABS = 1e-4


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    """||a - b|| / ||b||.  When the reference is (numerically) zero -- e.g. dQ
    of a single-key row, where dS = P (dP - D) = 0 exactly -- the ratio is
    meaningless; the denominator is floored at 1e-3 RMS so the max-abs bound
    decides."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    floor = 1e-3 * np.sqrt(max(b.size, 1))
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), floor))


def assert_bf16_close(name, got, ref, max_abs=BF16_MAX_ABS, rl2=BF16_REL_L2):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape, f"{name}: shape {got.shape} vs {ref.shape}"
    assert np.isfinite(got).all(), f"{name}: non-finite values"
    err = float(np.abs(got - ref).max()) if got.size else 0.0
    r = rel_l2(got, ref) if got.size else 0.0
    assert err <= max_abs and r <= rl2, f"{name}: max-abs {err:.3e} (<= {max_abs}), rel-L2 {r:.3e} (<= {rl2})"
    return err, r


def seeded_normal(shape, seed: int, device="cpu", dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(shape, generator=g, dtype=torch.float32).to(dtype).to(device)


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def assert_bf16_close_scaled(name, got, ref, tol=BF16_MAX_ABS, rl2=BF16_REL_L2):
    """bf16 outputs whose magnitude exceeds 1 (products, residual sums): the
    max-abs bound applies to |got - ref| / max(1, |ref|), i.e. absolute below
    1 and relative above (a bf16 output carries 2^-9 relative rounding)."""
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape, f"{name}: shape {got.shape} vs {ref.shape}"
    assert np.isfinite(got).all(), f"{name}: non-finite values"
    err = float((np.abs(got - ref) / np.maximum(1.0, np.abs(ref))).max()) if got.size else 0.0
    r = rel_l2(got, ref) if got.size else 0.0
    assert err <= tol and r <= rl2, f"{name}: scaled max-abs {err:.3e} (<= {tol}), rel-L2 {r:.3e} (<= {rl2})"
    return err, r

