"""Failure path of the attention kernels' bounded waits, exercised without a
GPU fault: a wait on a barrier that nothing arrives on gives up after the
limit (2 s), sets the CTA abort flag and the device status word, and the
context keeps working."""
import ctypes
import os
import subprocess
import time

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_bounded_wait_times_out_and_reports(cuda_device, tmp_path):
    so = str(tmp_path / "wait_timeout_probe.so")
    subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17",
                    "-Xcompiler", "-fPIC", "-shared", "-o", so,
                    os.path.join(HERE, "cuda", "wait_timeout_probe.cu")], check=True)
    lib = ctypes.CDLL(so)
    lib.wait_timeout_probe.argtypes = [ctypes.c_void_p]
    res = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    t0 = time.time()
    assert lib.wait_timeout_probe(ctypes.c_void_p(res.data_ptr())) == 0
    elapsed = time.time() - t0
    ok, abort_flag, status, after = res.cpu().tolist()
    assert ok == 0 and abort_flag == 1 and status == 77 and after == 1
    assert 1.5 < elapsed < 30


def test_peer_allreduce_barrier_times_out_and_reports(cuda_device):
    """The tensor-parallel all-reduce's cross-rank barrier, run as rank 0 of a
    2-rank group on one GPU where 'rank 1' is a local signal pad nothing ever
    writes: the flag wait gives up after its 2 s bound, the kernel returns,
    the device status holds the barrier's site code (801), and the context
    keeps working (a 1-rank call on the same buffers then completes)."""
    import teenyformers_b200 as tfb
    from teenyformers_b200 import _capi
    rows, cols = 256, 512
    pad_u32 = 256 + 2 * 128 * 8
    parts = [torch.randn(rows, cols, device=cuda_device).bfloat16() for _ in range(2)]
    hs = [torch.zeros(rows, cols, device=cuda_device, dtype=torch.bfloat16) for _ in range(2)]
    pads = [torch.zeros(pad_u32, device=cuda_device, dtype=torch.int32) for _ in range(2)]
    dev_ptrs = lambda ts: torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64,
                                       device=cuda_device)
    src, hp, sp = dev_ptrs(parts), dev_ptrs(hs), dev_ptrs(pads)
    p = lambda t: ctypes.c_void_p(0 if t is None else t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    assert tfb.device_status(clear=True) == 0
    t0 = time.time()
    _capi.call("tf_b200_allreduce_residual_rmsnorm_bf16", p(src), p(hp), p(sp), None, None, None,
               0, 2, rows, cols, 1e-5, 1, stream)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    assert tfb.device_status(clear=True) == 801
    assert 1.5 < elapsed < 30
    # the context is usable: a one-rank all-reduce (epoch 2) completes, h = partial
    _capi.call("tf_b200_allreduce_residual_rmsnorm_bf16", p(src), p(hp), p(sp), None, None, None,
               0, 1, rows, cols, 1e-5, 2, stream)
    torch.cuda.synchronize()
    assert tfb.device_status(clear=True) == 0
    assert torch.equal(hs[0], parts[0])
