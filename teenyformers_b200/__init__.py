"""teenyformers_b200 -- B200 (sm_100a) attention hot path for teenyformers.

Flash-attention-2 forward/backward (tcgen05 + TMA + TMEM), RoPE and the
head transpose/merge, behind the C ABI in include/teenyformers_b200.h.
The Python layer is a thin ctypes mirror of the reference op classes; the
native library is required (no CPU fallback).
"""
from . import _capi
from .ops import *  # noqa: F401,F403
from .ops import __all__ as _ops_all

__all__ = list(_ops_all) + ["library_path", "device_status"]

library_path = _capi.library_path
# The native library is loaded on first use; a missing library raises
# ImportError there (there is no fallback path).


def device_status(clear: bool = False) -> int:
    """Device-side error word (0 = no bounded wait ever timed out)."""
    return _capi.raw("tf_b200_device_status", int(bool(clear)))
