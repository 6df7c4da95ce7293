"""Host-side liveness of tensor-parallel ranks between steps.

A tensor-parallel step launches collectives (NCCL, and the peer-memory
exchanges inside the fused kernels) that only finish when every rank takes
part. A rank that has exited or stalled between steps would leave the others
waiting inside their next step's collectives. `RankWatch.step(i)` is called
by every rank before it launches step i: it records "rank r reached step i"
in a key-value store shared by the ranks (a torch.distributed Store) and
waits, bounded, until every rank has recorded step i. If a rank does not
arrive in time, the others raise `RankFailure` before launching anything of
step i; the caller then drops its communicator without the missing rank
(`CudaDevice.comm_abort`) instead of entering a collective that cannot
finish. This mirrors the reference's contract that a failed collective is a
`DeviceError::Execution` (docs/ARCH-0007 section 3), surfaced on the host.
"""
from __future__ import annotations

import datetime


class RankFailure(RuntimeError):
    """A rank did not reach the step in time (exited, stalled or hung)."""

    def __init__(self, step: int, missing: list[int], timeout_s: float):
        super().__init__(f"step {step}: rank(s) {missing} did not arrive within {timeout_s} s")
        self.step = step
        self.missing = missing


class RankWatch:
    """Per-step arrival check of `world` ranks through `store` (keys under
    `prefix`). Keys of steps older than the previous one are deleted, so the
    store holds at most two steps' keys."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0,
                 prefix: str = "slc/steps"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s = timeout_s
        self.prefix = prefix

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def step(self, i: int):
        """Records this rank's arrival at step i and waits for the others."""
        self.store.set(self._key(i, self.rank), "1")
        keys = [self._key(i, r) for r in range(self.world)]
        try:
            self.store.wait(keys, datetime.timedelta(seconds=self.timeout_s))
        except Exception:  # the store raises on timeout
            missing = [r for r, k in enumerate(keys) if not self.store.check([k])]
            raise RankFailure(i, missing, self.timeout_s) from None
        if i >= 2:
            try:
                self.store.delete_key(self._key(i - 2, self.rank))
            except Exception:
                pass
