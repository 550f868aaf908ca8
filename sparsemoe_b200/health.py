"""Host-side failure detection for the expert-parallel layer.

Every rank of an expert-parallel layer launches kernels and collectives that
the other ranks' memory or collectives complete.  A rank that has left (its
process raised, exited or was killed between steps) must therefore be noticed
on the host, before the next launch, rather than by a kernel or collective
that waits for it.  PeerWatch does that with the c10d key-value store the
process group already uses: before step s each rank publishes the key
`<prefix>/<rank>/<s>` and waits, with a wall-clock limit, for every peer's key
of the same step.  A peer that does not arrive in time raises PeerLost on the
survivors, with nothing of step s enqueued; the caller then tears down its
process group.  Nothing waits on the GPU.

The other half of the plan (a collective that is already in flight when a
peer dies) is the process group's own timeout: create the group with a short
`timeout=` so that its watchdog ends the collective with an error.
"""
from __future__ import annotations

import datetime


class PeerLost(RuntimeError):
    """A peer rank did not reach the current step within the limit."""

    def __init__(self, rank: int, step: int, missing: list[int], timeout_s: float):
        super().__init__(f"rank {rank}: peer rank(s) {missing} did not reach step {step} within {timeout_s:.1f} s")
        self.rank, self.step, self.missing = rank, step, missing


class PeerWatch:
    """Per-step liveness barrier over a c10d Store (host only, no GPU work).

    store:     the process group's store (`torch.distributed` default store,
               or any c10d Store shared by the ranks)
    rank, world: this rank and the group size
    timeout_s: how long a step waits for the slowest peer before declaring it
               lost; it bounds the host-side wait only
    """

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0, prefix: str = "sparsemoe_hb"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s = float(timeout_s)
        self.prefix = prefix
        self.step_no = 0

    @staticmethod
    def default_store():
        """The store behind torch.distributed's default process group."""
        import torch.distributed as dist
        return dist.distributed_c10d._get_default_store()

    def _key(self, rank: int, step: int) -> str:
        return f"{self.prefix}/{rank}/{step}"

    def step(self) -> int:
        """Announces this rank at the next step and waits for every peer to
        announce the same step; raises PeerLost naming the ranks that did not.
        Returns the step number."""
        s = self.step_no
        self.store.set(self._key(self.rank, s), b"1")
        peers = [r for r in range(self.world) if r != self.rank]
        keys = [self._key(r, s) for r in peers]
        try:
            if keys:
                self.store.wait(keys, datetime.timedelta(seconds=self.timeout_s))
        except Exception:   # the store raises on timeout (and on a dead store server)
            missing = [r for r in peers if not self._has(self._key(r, s))]
            raise PeerLost(self.rank, s, missing or peers, self.timeout_s) from None
        if s >= 2:          # keys two steps back are no longer waited on by anyone
            try:
                self.store.delete_key(self._key(self.rank, s - 2))
            except Exception:
                pass
        self.step_no = s + 1
        return s

    def _has(self, key: str) -> bool:
        try:
            return bool(self.store.check([key]))
        except Exception:
            return False
