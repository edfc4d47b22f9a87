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
