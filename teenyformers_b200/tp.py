"""Tensor-parallel all-reduce over NVLink peer memory, fused with the residual
add and RMSNorm that follow o_proj / down_proj in the Llama layer
(src/layers/llama_block.rs:55-65, fused_add_rmsnorm.rs:53-110).

`PeerAllReduceNorm` owns symmetric (peer-mapped) buffers from
torch.distributed._symmetric_memory -- torch is the allocator and the pointer
exchange here -- and launches ``tf_b200_allreduce_residual_rmsnorm_bf16``: one
kernel per call that reduce-scatters the ranks' partials with peer loads,
adds the residual, all-gathers h with peer stores and normalises locally.

Push mode (``pushed=True``): the producing GEMM (``ops.linear_push``) has
already stored each rank's rows into their owner's ``part`` buffer, read as
[world, rows / world, cols] (slot p = rank p's partial of this rank's rows),
while it ran; the kernel then sums those slots from local memory instead of
loading the partials over NVLink.
"""
from __future__ import annotations

import ctypes

import torch

from ._capi import call

_PAD_U32 = 256 + 2 * 128 * 8  # flags the kernel uses (offset + 2 phases x 128 CTAs x 8 ranks)


class PeerAllReduceNorm:
    """Symmetric [rows, cols] bf16 buffers for one tensor-parallel group.

    Use: write the rank's partial into ``part`` (e.g. ``torch.matmul(..., out=...)``),
    then ``h, y = ar(slot, residual, weight, eps)``; or push it with
    ``ops.linear_push(..., ar.recv_ptrs, rank, world)`` and call with ``pushed=True``.  ``h`` is a view of the
    symmetric h buffer ``slot`` (0 or 1): valid until the next call on that slot.
    Every rank must make the same calls in the same order.
    """

    def __init__(self, rows: int, cols: int, group=None, device=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if rows % self.world or cols % 8 or self.world > 8:
            raise ValueError("rows must split over the ranks, cols % 8 == 0, at most 8 ranks")
        self.rows, self.cols = rows, cols
        self.part = symm_mem.empty((rows, cols), dtype=torch.bfloat16, device=device)
        self.h = [symm_mem.empty((rows, cols), dtype=torch.bfloat16, device=device)
                  for _ in range(2)]
        self._hp = symm_mem.rendezvous(self.part, self.group)
        self._hh = [symm_mem.rendezvous(t, self.group) for t in self.h]
        if self._hp.signal_pad_size < _PAD_U32 * 4:
            raise RuntimeError("signal pad too small for the all-reduce flags")
        if self.part.data_ptr() != self._hp.buffer_ptrs[self.rank]:
            raise RuntimeError("symmetric buffer does not start at its allocation")
        self._hp.get_signal_pad(self._hp.rank, (_PAD_U32,), torch.int32).zero_()
        # push mode: every rank's receive buffer (host pointers, for the GEMM's
        # parameters) and, per slot p, this rank's own slot p shifted so that
        # global row r of slot p sits at src[p] + r * cols
        self.recv_ptrs = [int(p) for p in self._hp.buffer_ptrs]
        slice_bytes = (rows // self.world) * cols * 2
        base = self.part.data_ptr()
        self._local_src = torch.tensor(
            [base + (p - self.rank) * slice_bytes for p in range(self.world)], dtype=torch.int64,
            device=self.part.device)
        torch.cuda.synchronize(self.part.device)
        dist.barrier(self.group)
        self.epoch = 0

    def __call__(self, slot: int, residual: torch.Tensor | None, weight: torch.Tensor | None = None,
                 eps: float = 1e-5, y: torch.Tensor | None = None, pushed: bool = False):
        self.epoch += 1
        src = self._local_src.data_ptr() if pushed else self._hp.buffer_ptrs_dev
        h = self.h[slot]
        if weight is not None and y is None:
            y = torch.empty_like(h)
        ptr = lambda t: ctypes.c_void_p(0 if t is None else t.data_ptr())
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.part.device).cuda_stream)
        call("tf_b200_allreduce_residual_rmsnorm_bf16", ctypes.c_void_p(src),
             ctypes.c_void_p(self._hh[slot].buffer_ptrs_dev),
             ctypes.c_void_p(self._hp.signal_pad_ptrs_dev), ptr(residual), ptr(weight), ptr(y),
             self.rank, self.world, self.rows, self.cols, float(eps), self.epoch, stream)
        return h, y
