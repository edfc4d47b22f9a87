"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and rejects bad arguments before touching the device."""
import ctypes
import os
import re

import pytest

from teenyformers_b200 import _capi
from teenyformers_b200._capi import (TF_ERR_INVALID_ARG, TF_ERR_MISALIGNED, TF_ERR_UNSUPPORTED,
                                     TF_OK)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    syms = []
    for name in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if name.endswith(".h"):
            text = open(os.path.join(ROOT, "include", name)).read()
            syms += re.findall(r"^TF_API\s+[\w\s\*]+?\b(tf_b200_\w+)\s*\(", text, re.M)
    return syms


def test_header_declares_entry_points():
    syms = header_symbols()
    assert "tf_b200_flash_attn2_fwd_bf16" in syms and len(syms) >= 13


def test_library_exports_every_header_symbol(native_lib):
    for s in header_symbols():
        assert hasattr(native_lib, s), f"missing export {s}"
    assert set(header_symbols()) <= set(_capi.SIGNATURES), "ctypes table incomplete"


def test_version_and_status_strings(native_lib):
    assert native_lib.tf_b200_version() >= 1
    assert _capi.status_string(TF_ERR_MISALIGNED) == "misaligned pointer"


FAKE = ctypes.c_void_p(0x10000)      # 16-byte aligned, never dereferenced
ODD = ctypes.c_void_p(0x10002)       # misaligned for bf16 TMA


def fwd(*, q=FAKE, k=FAKE, v=FAKE, o=FAKE, lse=FAKE, B=1, Hq=2, Hkv=2, Sq=128, Sk=128, D=128,
        scale=0.1, causal=1):
    return _capi.raw("tf_b200_flash_attn2_fwd_bf16", q, k, v, o, lse, B, Hq, Hkv, Sq, Sk, D,
                     scale, causal, None)


def test_fwd_rejects_bad_arguments(native_lib):
    assert fwd(B=-1) == TF_ERR_INVALID_ARG
    assert fwd(D=96) == TF_ERR_UNSUPPORTED
    assert fwd(Hq=3, Hkv=2) == TF_ERR_UNSUPPORTED
    assert fwd(Sk=0) == TF_ERR_INVALID_ARG
    assert fwd(q=None) == TF_ERR_INVALID_ARG
    assert fwd(k=ODD) == TF_ERR_MISALIGNED
    assert fwd(scale=float("nan")) == TF_ERR_INVALID_ARG


def test_empty_problems_are_noops(native_lib):
    assert fwd(B=0, q=None) == TF_OK
    assert fwd(Sq=0) == TF_OK
    assert _capi.raw("tf_b200_transpose_heads", None, None, 0, 4, 2, 8, 2, None) == TF_OK
    assert _capi.raw("tf_b200_rope_bf16", None, None, 3, 0, 64, 9.2, 0, 0, None) == TF_OK


def test_bwd_workspace_size(native_lib):
    # -LSE*log2e and -D rows plus the fp32 dQ accumulator (128 columns), all
    # over B*Hq rows padded to a multiple of 128 queries, and a 256-byte
    # work-item counter
    n = _capi.raw("tf_b200_flash_attn2_bwd_workspace_size", 2, 3, 130)
    assert n == (2 + 128) * 2 * 3 * 256 * 4 + 256
    assert _capi.raw("tf_b200_flash_attn2_bwd_workspace_size", 0, 3, 130) == 0


def test_bwd_rejects_bad_arguments(native_lib):
    args = [FAKE] * 10 + [1, 4, 2, 64, 64, 128, 0.1, 1, None]
    bad = list(args)
    bad[9] = None  # workspace
    assert _capi.raw("tf_b200_flash_attn2_bwd_bf16", *bad) == TF_ERR_INVALID_ARG
    bad = list(args)
    bad[6] = ODD  # dq
    assert _capi.raw("tf_b200_flash_attn2_bwd_bf16", *bad) == TF_ERR_MISALIGNED
    bad = list(args)
    bad[15] = 80  # head_dim
    assert _capi.raw("tf_b200_flash_attn2_bwd_bf16", *bad) == TF_ERR_UNSUPPORTED


def test_rope_and_transpose_reject_bad_arguments(native_lib):
    assert _capi.raw("tf_b200_rope_bf16", FAKE, FAKE, 2, 8, 24, 9.2, 0, 0, None) == TF_ERR_UNSUPPORTED
    assert _capi.raw("tf_b200_rope_bf16", FAKE, FAKE, 2, 8, 64, 9.2, 7, 0, None) == TF_ERR_INVALID_ARG
    assert _capi.raw("tf_b200_rope_bf16", ODD, FAKE, 2, 8, 64, 9.2, 0, 0, None) == TF_ERR_MISALIGNED
    assert _capi.raw("tf_b200_rope_transpose_bf16", FAKE, FAKE, 1, 8, 2, 64, 9.2, 0, 0,
                     None) == TF_ERR_INVALID_ARG  # x == y
    assert _capi.raw("tf_b200_transpose_heads", FAKE, FAKE, 1, 4, 2, 8, 3, None) == TF_ERR_INVALID_ARG
    assert _capi.raw("tf_b200_merge_heads", FAKE, None, 1, 4, 2, 8, 2, None) == TF_ERR_INVALID_ARG


def test_gemm_entries_reject_bad_arguments(native_lib):
    g = lambda a, b, c, *rest: _capi.raw("tf_b200_gemm_bf16", a, b, None, c, *rest, None)
    assert g(FAKE, FAKE, FAKE, -1, 256, 64, 0) == TF_ERR_INVALID_ARG
    assert g(FAKE, FAKE, FAKE, 0, 256, 64, 0) == TF_OK          # empty output: no-op
    assert g(FAKE, FAKE, FAKE, 128, 256, 0, 0) == TF_ERR_UNSUPPORTED
    assert g(FAKE, FAKE, FAKE, 128, 256, 60, 0) == TF_ERR_UNSUPPORTED   # k % 8
    assert g(FAKE, FAKE, FAKE, 128, 250, 64, 0) == TF_ERR_UNSUPPORTED   # n % 8
    assert g(None, FAKE, FAKE, 128, 256, 64, 0) == TF_ERR_INVALID_ARG
    assert g(FAKE, FAKE, ODD, 128, 256, 64, 0) == TF_ERR_MISALIGNED
    assert g(FAKE, FAKE, FAKE, 256, 256, 192, 128) == TF_ERR_UNSUPPORTED  # heads layout: k % 128
    assert g(FAKE, FAKE, FAKE, 384, 256, 256, 256) == TF_ERR_UNSUPPORTED  # m % a_seq
    sw = lambda *a: _capi.raw("tf_b200_gemm_swiglu_bf16", *a, None)
    assert sw(FAKE, FAKE, FAKE, 128, 200, 64) == TF_ERR_UNSUPPORTED      # d_ff % 128
    assert sw(FAKE, FAKE, None, 128, 256, 64) == TF_ERR_INVALID_ARG
    qkv = lambda *a: _capi.raw("tf_b200_gemm_qkv_rope_bf16", *a, None)
    assert qkv(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 1, 200, 2, 1, 256, 0) == TF_ERR_UNSUPPORTED
    assert qkv(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 1, 256, 2, 1, 256, 5) == TF_ERR_INVALID_ARG
    assert qkv(FAKE, FAKE, FAKE, None, FAKE, FAKE, 1, 256, 2, 1, 256, 0) == TF_ERR_INVALID_ARG
    assert qkv(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 0, 256, 2, 1, 256, 0) == TF_OK
    assert _capi.raw("tf_b200_rope_table_f32", FAKE, 16, 7, 9.2, None) == TF_ERR_INVALID_ARG
    peers = (ctypes.c_void_p * 2)(0x10000, 0x20000)
    push = lambda *a: _capi.raw("tf_b200_gemm_push_bf16", *a, None)
    assert push(FAKE, FAKE, peers, 512, 256, 64, 0, 0, 9) == TF_ERR_INVALID_ARG   # world > 8
    assert push(FAKE, FAKE, peers, 512, 256, 64, 0, 2, 2) == TF_ERR_INVALID_ARG   # rank
    assert push(FAKE, FAKE, peers, 384, 256, 64, 0, 0, 2) == TF_ERR_UNSUPPORTED   # slice % 128
    assert push(FAKE, FAKE, None, 512, 256, 64, 0, 0, 2) == TF_ERR_INVALID_ARG
    odd = (ctypes.c_void_p * 2)(0x10000, 0x20002)
    assert push(FAKE, FAKE, odd, 512, 256, 64, 0, 0, 2) == TF_ERR_MISALIGNED


def test_op_shape_inference_mirrors_reference():
    from teenyformers_b200 import (CausalFlashAttn2Op, FlashAttn2Op, MergeHeadsOp, RopeOp,
                                   TransposeHeadsOp)
    op = CausalFlashAttn2Op(64, 0.125)
    assert op.name == "causal_flash_attn2" and FlashAttn2Op(64, 0.1).name == "flash_attn2"
    assert op.infer_output_shape([(8, 100, 64), (8, 120, 64), (8, 120, 64)]) == (8, 100, 64)
    assert op.param_shapes([(8, 100, 64)]) == [[8, 100]]  # l cache [BH, Nq]
    assert op.n_activation_inputs() == 3
    assert RopeOp(64, 1e4).param_shapes([(2, 3, 64)]) == []
    assert TransposeHeadsOp(4, 16).infer_output_shape([(10, 64)]) == (4, 10, 16)
    assert MergeHeadsOp(4, 16).infer_output_shape([(4, 10, 16)]) == (10, 64)


def test_backward_size_limits_reject_without_overflow(native_lib):
    """Head counts whose products would overflow 64-bit arithmetic are refused
    before any device work (workspace size 0, TF_ERR_TOO_LARGE)."""
    big = 1 << 30
    assert _capi.raw("tf_b200_flash_attn2_bwd_workspace_size", big, big, 4096) == 0
    assert _capi.raw("tf_b200_flash_attn2_bwd_workspace_size", 1, 1, 1) > 0
    args = [FAKE] * 9
    rc = _capi.raw("tf_b200_flash_attn2_bwd_bf16", *args, FAKE, big, big, big, 1 << 20,
                   1 << 20, 128, 0.1, 1, None)
    assert rc == _capi.TF_ERR_TOO_LARGE
    for B, H, S in ((big, big, 4096), (1, 257, 4096), (1, 1, 1 << 30)):
        rc = _capi.raw("tf_b200_flash_attn2_bwd_bf16_noalloc", *args, B, H, H, S, S, 128, 0.1, 1,
                       None)
        assert rc == _capi.TF_ERR_TOO_LARGE, (B, H, S)


# C parameter type in the header -> its declaration in the Rust binding
_C_TO_RUST = {
    "const void*": "*const c_void", "void*": "*mut c_void", "const float*": "*const f32",
    "float*": "*mut f32", "int": "c_int", "float": "f32", "size_t": "usize", "unsigned": "u32",
    "const int*": "*const c_int", "const char*": "*const c_char",
    "const void* const*": "*const *const c_void", "void* const*": "*const *mut c_void",
}


def _header_decls():
    out = {}
    for name in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not name.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", name)).read()
        for d in re.findall(r"^TF_API\s+([^;]*?\))\s*;", text, re.M | re.S):
            d = " ".join(d.split())
            m = re.match(r"(.+?)\b(tf_b200_\w+)\((.*)\)$", d)
            params = []
            if m.group(3) != "void":
                for p in m.group(3).split(","):
                    pm = re.match(r"(.*?)(\w+)$", p.strip())
                    params.append((pm.group(2), _C_TO_RUST[pm.group(1).strip().replace(" *", "*")]))
            out[m.group(2)] = (_C_TO_RUST[m.group(1).strip()], params)
    return out


def test_rust_binding_matches_header():
    """rust/teeny-b200-sys declares every header entry point with the same
    parameter names and types, in order (the crate is not compiled here)."""
    src = open(os.path.join(ROOT, "rust", "teeny-b200-sys", "src", "lib.rs")).read()
    block = src[src.index('unsafe extern "C" {'):]
    block = block[:block.index("\n    }\n")]
    rust = {}
    for m in re.finditer(r"pub fn (tf_b200_\w+)\((.*?)\)\s*->\s*([^;]+);", block, re.S):
        params = []
        for p in " ".join(m.group(2).split()).split(","):
            p = p.strip()
            if p:
                n, t = p.split(":", 1)
                params.append((n.strip(), t.strip()))
        rust[m.group(1)] = (m.group(3).strip(), params)
    header = _header_decls()
    assert set(rust) == set(header), set(rust) ^ set(header)
    for name, decl in header.items():
        assert rust[name] == decl, name
    toml = open(os.path.join(ROOT, "rust", "teeny-b200-sys", "Cargo.toml")).read()
    assert 'links = "teenyformers_b200"' in toml
