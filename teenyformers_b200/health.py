"""Host-side detection of a rank that left the tensor-parallel group.

The multi-GPU paths here (the config #5 layer's all-reduces, the bench's
max-over-ranks timing) assume every rank takes the same collective steps.  If
one rank stops between steps -- it raised, was killed, or never reached the
step -- the others would otherwise block inside their next collective until
the process-group timeout.  ``StepHeartbeat`` lets each rank publish the step
it has reached in the process group's key-value store and check, before it
launches the next step's kernels and collectives, that every peer has reached
the previous one; a peer that has not within ``timeout`` seconds raises
``RankFailure`` on the host, with no kernel or collective of that step in
flight.  Nothing here touches the GPU.
"""
from __future__ import annotations

import time


class RankFailure(RuntimeError):
    """A peer did not reach a step in time (it left, or is stalled)."""

    def __init__(self, rank: int, step: int, missing: list):
        super().__init__(f"rank {rank}: peers {missing} did not reach step {step}")
        self.missing = missing
        self.step = step


class StepHeartbeat:
    """Per-step presence flags in a torch.distributed Store.

    Each step starts with ``beat(step)`` (this rank is present for the step)
    and ``check(step)`` (so is every other rank) before the step's kernels and
    collectives are launched.
    """

    def __init__(self, store, rank: int, world: int, timeout: float = 10.0,
                 prefix: str = "tfb_hb"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout = float(timeout)
        self.prefix = prefix

    def _key(self, rank: int, step: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def beat(self, step: int) -> None:
        self.store.set(self._key(self.rank, step), "1")

    def check(self, step: int) -> None:
        """Returns once every rank has beaten ``step``; raises RankFailure
        naming the ranks that have not within the timeout."""
        keys = [self._key(r, step) for r in range(self.world)]
        deadline = time.monotonic() + self.timeout
        while True:
            missing = [r for r, k in enumerate(keys) if not self.store.check([k])]
            if not missing:
                return
            if time.monotonic() >= deadline:
                raise RankFailure(self.rank, step, missing)
            time.sleep(0.01)
