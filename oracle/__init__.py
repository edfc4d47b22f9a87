"""CPU oracle for teenyformers' attention path -- TEST INFRASTRUCTURE ONLY.

Thin numpy/ctypes wrapper over ``oracle/liboracle.so`` (built from
``oracle/oracle.c`` by ``oracle/Makefile``).  Each function restates a
reference kernel in fp32; see the citations in ``oracle.c``.  Only tests,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import this
package; the product library never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

ROPE_INTERLEAVED = 0
ROPE_ROTATE_HALF = 1


def build() -> str:
    """Compile liboracle.so in place (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
        os.path.join(_HERE, "oracle.c")
    ):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    P = ctypes.c_void_p
    I = ctypes.c_int
    F = ctypes.c_float
    lib.orc_flash_attn2_fwd_range.argtypes = [P] * 5 + [I] * 6 + [F, I] + [I] * 4
    lib.orc_flash_attn2_fwd.argtypes = [P] * 5 + [I] * 6 + [F, I]
    lib.orc_flash_attn2_bwd.argtypes = [P] * 9 + [I] * 6 + [F, I]
    lib.orc_rope.argtypes = [P, P, I, I, I, F, I, I]
    lib.orc_transpose_heads.argtypes = [P, P, I, I, I, I, I]
    lib.orc_merge_heads.argtypes = [P, P, I, I, I, I, I]
    lib.orc_rope_transpose.argtypes = [P, P, I, I, I, I, F, I, I]
    lib.orc_rmsnorm.argtypes = [P, P, P, P, P, I, I, F]
    lib.orc_swiglu.argtypes = [P, P, I, I]
    lib.orc_max_threads.restype = I
    lib.orc_set_threads.argtypes = [I]
    _lib = lib
    return lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def max_threads() -> int:
    return _load().orc_max_threads()


def set_threads(n: int) -> None:
    _load().orc_set_threads(int(n))


def flash_attn2_fwd(q, k, v, scale: float, causal: bool, n_heads_kv: int | None = None,
                    bh_range=None, q_range=None):
    """q [B,Hq,Sq,D], k/v [B,Hkv,Sk,D] (or 3-D [BH,S,D]) -> (o, lse).

    With ``bh_range``/``q_range`` only that block of rows is computed (the
    rest of ``o``/``lse`` is left as NaN) -- a bounded sample for timing.
    """
    q, k, v = _f32(q), _f32(k), _f32(v)
    if q.ndim == 3:
        q, k, v = q[None], k[None], v[None]
    B, Hq, Sq, D = q.shape
    Hkv = k.shape[1] if n_heads_kv is None else n_heads_kv
    Sk = k.shape[2]
    o = np.full(q.shape, np.nan, dtype=np.float32)
    lse = np.full((B, Hq, Sq), np.nan, dtype=np.float32)
    bh_lo, bh_hi = bh_range if bh_range is not None else (0, B * Hq)
    q_lo, q_hi = q_range if q_range is not None else (0, Sq)
    _load().orc_flash_attn2_fwd_range(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), B, Hq,
                                      Hkv, Sq, Sk, D, float(scale), int(bool(causal)),
                                      bh_lo, bh_hi, q_lo, q_hi)
    return o, lse


def flash_attn2_bwd(q, k, v, o, do, lse, scale: float, causal: bool):
    """Gradients (dq, dk, dv) of the reference backward, same layouts as fwd."""
    q, k, v, o, do, lse = (_f32(x) for x in (q, k, v, o, do, lse))
    squeeze = q.ndim == 3
    if squeeze:
        q, k, v, o, do = q[None], k[None], v[None], o[None], do[None]
        lse = lse[None]
    B, Hq, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    _load().orc_flash_attn2_bwd(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(do), _ptr(lse),
                                _ptr(dq), _ptr(dk), _ptr(dv), B, Hq, Hkv, Sq, Sk, D,
                                float(scale), int(bool(causal)))
    if squeeze:
        return dq[0], dk[0], dv[0]
    return dq, dk, dv


def rope(x, ln_base: float, style: int = ROPE_INTERLEAVED, inverse: bool = False):
    """RoPE on [BH, S, D] (or [..., S, D]); pos = index along S."""
    x = _f32(x)
    S, D = x.shape[-2], x.shape[-1]
    BH = int(np.prod(x.shape[:-2])) if x.ndim > 2 else 1
    y = np.empty_like(x)
    _load().orc_rope(_ptr(x), _ptr(y), BH, S, D, float(ln_base), int(style), int(bool(inverse)))
    return y


def transpose_heads(src, n_heads: int):
    """[B, S, H*D] or [B, S, H, D] -> [B, H, S, D]; any dtype, bit-exact copy."""
    src = np.ascontiguousarray(src)
    B, S = src.shape[0], src.shape[1]
    D = (src.shape[2] // n_heads) if src.ndim == 3 else src.shape[3]
    dst = np.empty((B, n_heads, S, D), dtype=src.dtype)
    _load().orc_transpose_heads(_ptr(src), _ptr(dst), B, S, n_heads, D, src.dtype.itemsize)
    return dst


def merge_heads(src):
    """[B, H, S, D] -> [B, S, H, D]; any dtype, bit-exact copy."""
    src = np.ascontiguousarray(src)
    B, H, S, D = src.shape
    dst = np.empty((B, S, H, D), dtype=src.dtype)
    _load().orc_merge_heads(_ptr(src), _ptr(dst), B, S, H, D, src.dtype.itemsize)
    return dst


def rope_transpose(x, ln_base: float, style: int = ROPE_INTERLEAVED, inverse: bool = False):
    """Forward: x [B,S,H,D] -> RoPE(transpose(x)) [B,H,S,D].
    Inverse: dy [B,H,S,D] -> merge(RoPE^-1(dy)) [B,S,H,D]."""
    x = _f32(x)
    if not inverse:
        B, S, H, D = x.shape
        y = np.empty((B, H, S, D), dtype=np.float32)
    else:
        B, H, S, D = x.shape
        y = np.empty((B, S, H, D), dtype=np.float32)
    _load().orc_rope_transpose(_ptr(x), _ptr(y), B, S, H, D, float(ln_base), int(style),
                               int(bool(inverse)))
    return y


def rmsnorm(x, weight, eps: float, residual=None):
    """(y, h): h = x + residual (or x), y = h * rsqrt(mean(h^2) + eps) * weight."""
    x = _f32(x)
    N = x.shape[-1]
    M = x.size // N if N else 0
    w = _f32(weight)
    r = _f32(residual) if residual is not None else None
    y = np.empty_like(x)
    h = np.empty_like(x)
    _load().orc_rmsnorm(_ptr(x), _ptr(r) if r is not None else None, _ptr(w), _ptr(y), _ptr(h),
                        M, N, float(eps))
    return y, h


def swiglu(z):
    """z [..., 2*d_ff] = gate || up -> silu(gate) * up [..., d_ff]."""
    z = _f32(z)
    d_ff = z.shape[-1] // 2
    M = z.size // (2 * d_ff) if d_ff else 0
    out = np.empty(z.shape[:-1] + (d_ff,), dtype=np.float32)
    _load().orc_swiglu(_ptr(z), _ptr(out), M, d_ff)
    return out
