"""The allocation-free backward entry point, through the C ABI.

Some callers cannot hand the backward a scratch buffer: an executor that
sizes every device buffer up front from the ops' declared shapes (the
reference's passes a backward exactly q, k, v, o, dO, l, dq, dk, dv), or a
process that may not allocate once running.  tf_b200_flash_attn2_bwd_bf16_noalloc
keeps its scratch in a fixed array inside the library instead.  This file is
collected last so a failure here leaves every other test already run."""
import ctypes

import pytest
import torch

from teenyformers_b200 import _capi
from tests.helpers import assert_bf16_close, seeded_normal, to_np

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _run_both(dev, B, Hq, Hkv, Sq, Sk, D, causal, seed, calls=2):
    """Backward through the workspace entry point, then `calls` times through
    the allocation-free one; every allocation-free result must match."""
    scale = D ** -0.5
    q = seeded_normal((B, Hq, Sq, D), seed, device=dev)
    k = seeded_normal((B, Hkv, Sk, D), seed + 1, device=dev)
    v = seeded_normal((B, Hkv, Sk, D), seed + 2, device=dev)
    do = seeded_normal((B, Hq, Sq, D), seed + 3, device=dev)
    o = torch.empty_like(q)
    lse = torch.empty((B, Hq, Sq), dtype=torch.float32, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    _capi.call("tf_b200_flash_attn2_fwd_bf16", _p(q), _p(k), _p(v), _p(o), _p(lse), B, Hq, Hkv,
               Sq, Sk, D, scale, int(causal), stream)
    # reference result: the entry point that takes a caller workspace
    n_ws = _capi.raw("tf_b200_flash_attn2_bwd_workspace_size", B, Hq, Sq)
    ws = torch.empty(n_ws, dtype=torch.uint8, device=dev)
    ref = [torch.empty_like(t) for t in (q, k, v)]
    _capi.call("tf_b200_flash_attn2_bwd_bf16", _p(q), _p(k), _p(v), _p(o), _p(do), _p(lse),
               *(_p(t) for t in ref), _p(ws), B, Hq, Hkv, Sq, Sk, D, scale, int(causal), stream)
    for call in range(calls):
        got = [torch.full_like(t, float("nan")) for t in (q, k, v)]
        _capi.call("tf_b200_flash_attn2_bwd_bf16_noalloc", _p(q), _p(k), _p(v), _p(o), _p(do),
                   _p(lse), *(_p(t) for t in got), B, Hq, Hkv, Sq, Sk, D, scale, int(causal),
                   stream)
        torch.cuda.synchronize()
        for name, a, b in zip(("dq", "dk", "dv"), got, ref):
            assert_bf16_close(f"{name} (call {call}, Sq={Sq} Sk={Sk})", to_np(a), to_np(b))


def test_noalloc_backward_matches_workspace_backward_twice(cuda_device):
    _run_both(cuda_device, 2, 8, 4, 640, 640, 128, True, seed=31)


def test_noalloc_backward_after_a_larger_call_ragged_shapes(cuda_device):
    """The array keeps the previous call's contents: a large call first, then
    ragged calls (Sq not a multiple of 128, so the array's padded rows are
    used, and Sq != Sk), causal and not, each against the workspace path."""
    _run_both(cuda_device, 4, 16, 16, 2048, 2048, 128, True, seed=41, calls=1)
    _run_both(cuda_device, 1, 4, 2, 77, 200, 128, True, seed=51)
    _run_both(cuda_device, 1, 4, 2, 77, 200, 64, False, seed=61)
    _run_both(cuda_device, 2, 2, 1, 300, 130, 128, True, seed=71)


def test_noalloc_backward_rejects_sizes_beyond_its_array(cuda_device):
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: rejected before any launch
    # 1 x 300 heads x 4096 rows > the 1,048,576 rows the array holds
    rc = _capi.raw("tf_b200_flash_attn2_bwd_bf16_noalloc", *([fake] * 9), 1, 300, 300, 4096,
                   4096, 128, 0.088, 1, None)
    assert rc == _capi.TF_ERR_TOO_LARGE
