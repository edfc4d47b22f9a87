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


def test_noalloc_backward_matches_workspace_backward_twice(cuda_device):
    B, Hq, Hkv, S, D = 2, 8, 4, 640, 128
    scale = D ** -0.5
    q = seeded_normal((B, Hq, S, D), 31, device=cuda_device)
    k = seeded_normal((B, Hkv, S, D), 32, device=cuda_device)
    v = seeded_normal((B, Hkv, S, D), 33, device=cuda_device)
    do = seeded_normal((B, Hq, S, D), 34, device=cuda_device)
    o = torch.empty_like(q)
    lse = torch.empty((B, Hq, S), dtype=torch.float32, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    _capi.call("tf_b200_flash_attn2_fwd_bf16", _p(q), _p(k), _p(v), _p(o), _p(lse), B, Hq, Hkv,
               S, S, D, scale, 1, stream)
    # reference result: the entry point that takes a caller workspace
    n_ws = _capi.raw("tf_b200_flash_attn2_bwd_workspace_size", B, Hq, S)
    ws = torch.empty(n_ws, dtype=torch.uint8, device=cuda_device)
    ref = [torch.empty_like(t) for t in (q, k, v)]
    _capi.call("tf_b200_flash_attn2_bwd_bf16", _p(q), _p(k), _p(v), _p(o), _p(do), _p(lse),
               *(_p(t) for t in ref), _p(ws), B, Hq, Hkv, S, S, D, scale, 1, stream)
    # two calls in a row through the allocation-free entry point
    for call in range(2):
        got = [torch.full_like(t, float("nan")) for t in (q, k, v)]
        _capi.call("tf_b200_flash_attn2_bwd_bf16_noalloc", _p(q), _p(k), _p(v), _p(o), _p(do),
                   _p(lse), *(_p(t) for t in got), B, Hq, Hkv, S, S, D, scale, 1, stream)
        torch.cuda.synchronize()
        for name, a, b in zip(("dq", "dk", "dv"), got, ref):
            assert_bf16_close(f"{name} (call {call})", to_np(a), to_np(b))


def test_noalloc_backward_rejects_sizes_beyond_its_array(cuda_device):
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: rejected before any launch
    # 1 x 300 heads x 4096 rows > the 1,048,576 rows the array holds
    rc = _capi.raw("tf_b200_flash_attn2_bwd_bf16_noalloc", *([fake] * 9), 1, 300, 300, 4096,
                   4096, 128, 0.088, 1, None)
    assert rc == _capi.TF_ERR_TOO_LARGE
