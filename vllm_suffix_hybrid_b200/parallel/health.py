"""Host-side failure detection for ranks that step in lockstep (tensor / expert parallel serving).

The ranks share one flag in the process group's rendezvous store.  A rank whose step raises records
(rank, reason) in the flag before it leaves; every rank tests the flag between steps (a non-blocking key
test on the store) and stops with `RankFailure` naming the failed rank instead of entering a collective that
would wait for it.  A rank that dies without recording anything (killed) is caught by the short timeout of
the next collective, whose error is reported as `RankFailure` too, with the flag's contents when a peer did
record one.  Detection runs on the host between steps, with no kernel or collective of this rank in flight.

The reference has no counterpart: its host all-reduce barrier traps after a spin budget
(reference: suffix_hybrid/host_ar.py:148-166); here device waits return error codes and rank loss is
reported on the host.
"""
from __future__ import annotations

import logging
from typing import Optional

logger = logging.getLogger(__name__)

KEY = "suffix_hybrid/health/failed"


class RankFailure(RuntimeError):
    """A peer rank failed (or left); `rank` is the failed rank when it recorded itself, else -1."""

    def __init__(self, message: str, rank: int = -1):
        super().__init__(message)
        self.rank = rank


class RankHealth:
    """The shared failure flag of one process group; a no-op for a single rank."""

    def __init__(self, store=None, rank: int = 0, world: int = 1, every: int = 1):
        self.store = store if world > 1 else None
        self.rank, self.world = rank, world
        self.every = max(1, int(every))
        self._n = 0

    @classmethod
    def from_process_group(cls, every: int = 1) -> "RankHealth":
        """The flag in the default process group's store (the torchrun rendezvous store)."""
        import torch.distributed as dist

        if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
            return cls()
        from torch.distributed import distributed_c10d

        return cls(distributed_c10d._get_default_store(), dist.get_rank(), dist.get_world_size(), every)

    def report(self, reason: str) -> None:
        """Record this rank as failed (the first record wins); never raises."""
        if self.store is None:
            return
        try:
            if not self.store.check([KEY]):
                self.store.set(KEY, f"{self.rank}|{reason[:400]}")
        except Exception:  # the store itself may be gone; the peers' collective timeout still fires
            logger.warning("rank %d: could not record its failure in the store", self.rank)

    def failed(self) -> Optional[tuple]:
        """(rank, reason) of a recorded failure, or None."""
        if self.store is None or not self.store.check([KEY]):
            return None
        raw = self.store.get(KEY).decode(errors="replace")
        r, _, why = raw.partition("|")
        return (int(r) if r.lstrip("-").isdigit() else -1), why

    def check(self) -> None:
        """Raise RankFailure if a rank recorded a failure (tested every `every` calls)."""
        if self.store is None:
            return
        self._n += 1
        if self._n % self.every:
            return
        f = self.failed()
        if f is not None and f[0] != self.rank:
            raise RankFailure(f"rank {f[0]} failed: {f[1]}", f[0])

    def explain(self, err: BaseException) -> RankFailure:
        """The RankFailure for a collective that raised `err` (a peer's record if there is one)."""
        f = None
        try:
            f = self.failed()
        except Exception:
            pass
        if f is not None:
            return RankFailure(f"rank {f[0]} failed: {f[1]} (collective error: {err!r})", f[0])
        return RankFailure(f"a collective failed and no rank recorded a failure (a peer left?): {err!r}")
