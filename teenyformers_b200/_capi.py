"""ctypes binding of include/teenyformers_b200.h.

Loads the in-tree ``lib/libteenyformers_b200.so``.  There is no fallback: if
the library is missing or does not export a symbol, import fails loudly.
"""
from __future__ import annotations

import ctypes
import os

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib",
                         "libteenyformers_b200.so")

TF_OK = 0
TF_ERR_INVALID_ARG = -1
TF_ERR_UNSUPPORTED = -2
TF_ERR_MISALIGNED = -3
TF_ERR_CUDA = -4
TF_ERR_TOO_LARGE = -5
TF_ERR_DEVICE_TIMEOUT = -6

TF_ROPE_INTERLEAVED = 0
TF_ROPE_ROTATE_HALF = 1

P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float
SZ = ctypes.c_size_t

# name -> (restype, argtypes), in header order
SIGNATURES = {
    "tf_b200_version": (I, []),
    "tf_b200_status_string": (ctypes.c_char_p, [I]),
    "tf_b200_device_status": (I, [I]),
    "tf_b200_flash_attn2_fwd_bf16": (I, [P, P, P, P, P, I, I, I, I, I, I, F, I, P]),
    "tf_b200_flash_attn2_bwd_workspace_size": (SZ, [I, I, I]),
    "tf_b200_flash_attn2_bwd_bf16": (I, [P] * 10 + [I, I, I, I, I, I, F, I, P]),
    "tf_b200_flash_attn2_bwd_bf16_noalloc": (I, [P] * 9 + [I, I, I, I, I, I, F, I, P]),
    "tf_b200_flash_attn2_decode_workspace_size": (SZ, [I] * 6),
    "tf_b200_flash_attn2_decode_bf16": (I, [P] * 6 + [I] * 6 + [F, P, P]),
    "tf_b200_allreduce_residual_rmsnorm_bf16": (I, [P] * 6 + [I] * 4 + [F, ctypes.c_uint, P]),
    "tf_b200_flash_attn2_fwd_f32": (I, [P, P, P, P, P, I, I, I, I, F, F, I, P]),
    "tf_b200_flash_attn2_bwd_f32": (I, [P] * 9 + [I, I, I, I, F, I, P]),
    "tf_b200_rope_f32": (I, [P, P, I, I, I, F, I, I, P]),
    "tf_b200_rope_bf16": (I, [P, P, I, I, I, F, I, I, P]),
    "tf_b200_rope_transpose_bf16": (I, [P, P, I, I, I, I, F, I, I, P]),
    "tf_b200_transpose_heads": (I, [P, P, I, I, I, I, I, P]),
    "tf_b200_merge_heads": (I, [P, P, I, I, I, I, I, P]),
    "tf_b200_rmsnorm_bf16": (I, [P, P, P, P, P, I, I, F, P]),
    "tf_b200_swiglu_bf16": (I, [P, P, I, I, P]),
    "tf_b200_gemm_bf16": (I, [P, P, P, P, I, I, I, I, P]),
    "tf_b200_gemm_swiglu_bf16": (I, [P, P, P, I, I, I, P]),
    "tf_b200_rope_table_f32": (I, [P, I, I, F, P]),
    "tf_b200_gemm_qkv_rope_bf16": (I, [P] * 6 + [I] * 6 + [P]),
    "tf_b200_gemm_push_bf16": (I, [P, P, ctypes.POINTER(ctypes.c_void_p)] + [I] * 6 + [P]),
}


class TfError(RuntimeError):
    def __init__(self, fn: str, code: int):
        self.code = code
        super().__init__(f"{fn} failed: {code} ({status_string(code)})")


def library_path() -> str:
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise ImportError(
                f"teenyformers_b200 native library not built: {_LIB_PATH} "
                "(run `python -m teenyformers_b200.build`)")
        handle = ctypes.CDLL(_LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)  # AttributeError if the export is missing
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def status_string(code: int) -> str:
    return lib().tf_b200_status_string(int(code)).decode()


def call(name: str, *args) -> int:
    """Calls an int-returning entry point; raises TfError on a negative status."""
    rc = getattr(lib(), name)(*args)
    if rc != TF_OK:
        raise TfError(name, rc)
    return rc


def raw(name: str, *args):
    """Calls an entry point and returns its raw result (no error check)."""
    return getattr(lib(), name)(*args)
