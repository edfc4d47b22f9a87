"""Builds the in-tree native library for sm_100a.

    python -m teenyformers_b200.build

Produces ``teenyformers_b200/lib/libteenyformers_b200.so`` from
``teenyformers_b200/csrc/tfb_lib.cu`` (one nvcc invocation; cudart linked
statically so the library has no runtime dependency beyond the driver), and
the C++ op-layer check program ``teenyformers_b200/lib/ops_selftest``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libteenyformers_b200.so")
SELFTEST = os.path.join(LIBDIR, "ops_selftest")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                           "-Xcompiler", "-fvisibility=hidden"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))] + [
        os.path.join(ROOT, "include", "teenyformers_b200.h"),
        os.path.join(ROOT, "include", "teenyformers_b200_ops.hpp"),
    ]


def _stale(target: str) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.exists(s) and os.path.getmtime(s) > t for s in _sources())


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    if force or _stale(LIB):
        cmd = [nvcc()] + NVCC_FLAGS + ["-shared", "-o", LIB, os.path.join(CSRC, "tfb_lib.cu")]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    ops_test = os.path.join(CSRC, "ops_selftest.cpp")
    if os.path.exists(ops_test) and (force or _stale(SELFTEST)):
        cmd = ["g++", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"),
               "-I", "/usr/local/cuda/include", ops_test, "-o", SELFTEST,
               "-L", LIBDIR, "-lteenyformers_b200", "-Wl,-rpath,$ORIGIN",
               "-L", "/usr/local/cuda/lib64", "-lcudart"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
