"""Host-side failure detection for tensor-parallel decoding.

Under tensor parallelism every decode step ends in collectives that need all
ranks: a rank that has stopped (crashed, was killed, left the loop) leaves
the others' NCCL kernels waiting.  Two layers catch that:

* in the runtime, every synchronous call and every step of the asynchronous
  decode waits for its work with a bound (`collective_timeout_ms` model
  option); on expiry it aborts the NCCL communicator, so the kernels return,
  and reports WL_ERR_TIMEOUT (the model must then be closed and reloaded);
* here, before each step a rank publishes a heartbeat (its step number) in a
  torch.distributed key-value store and checks that every other rank has
  reached the previous step, with a short timeout.  A rank that left between
  steps is thus noticed on the host before anyone enters the collective that
  could never complete; the caller gets WoollyError(WL_ERR_NCCL) naming the
  missing ranks, and can abort the communicator (abort_communicator).

The reference has no multi-process path; its error kinds are the CoreError
codes (woolly-core/src/lib.rs:30-165), which WoollyError mirrors.
"""
from __future__ import annotations

import time

from ._lib import WL_ERR_NCCL, WoollyError, check, lib


class RankWatch:
    """Heartbeats of the ranks of one tensor-parallel group in a Store."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, prefix: str = "wl_tp"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s = timeout_s
        self.prefix = prefix
        self.step = -1

    def _key(self, r: int) -> str:
        return f"{self.prefix}/beat/{r}"

    def beat(self, step: int) -> None:
        """This rank is about to run step `step`."""
        self.step = step
        self.store.set(self._key(self.rank), str(step))

    def leave(self) -> None:
        """This rank stops participating (marks itself gone for the others)."""
        self.store.set(self._key(self.rank), "-1")

    def missing(self, step: int) -> list[int]:
        """Ranks that have not reached `step` (or have left)."""
        out = []
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                v = int(self.store.get(self._key(r)))
            except Exception:
                v = -2
            if v < step:
                out.append(r)
        return out

    def check(self, step: int) -> None:
        """Waits (bounded) until every rank has announced `step`; raises
        WoollyError(WL_ERR_NCCL) with the missing ranks otherwise."""
        t0 = time.monotonic()
        while True:
            miss = self.missing(step)
            if not miss:
                return
            if time.monotonic() - t0 > self.timeout_s:
                raise WoollyError(WL_ERR_NCCL,
                                  f"tensor-parallel ranks {miss} did not reach step {step} within "
                                  f"{self.timeout_s:.1f} s: not entering the collective")
            time.sleep(0.005)

    def guard(self, step: int) -> None:
        """beat(step) then check(step): call before launching a step."""
        self.beat(step)
        self.check(step)


def abort_communicator(comm: int) -> None:
    """ncclCommAbort on a communicator made by model.nccl_communicator."""
    import ctypes as C
    check(lib().wl_nccl_comm_abort(C.c_void_p(comm)))
