"""Host-side liveness of a job's ranks, through the process group's key-value store.

Every device wait in the expert-parallel kernels is bounded, and a short process-group
timeout ends a collective whose peer is gone. Both notice a lost rank only after work
has been launched against it. ``Heartbeat`` lets the ranks learn it on the host first,
between steps, so a rank that is gone (crashed, killed, hung on the host, or drained on
purpose) is reported by name before anyone launches kernels that would wait for it.

* ``arrive(step)`` at the start of every step (0-based): this rank's counter in the store
  goes up by one (``store.add``, atomic; no clock is compared across hosts), then it
  waits until every peer has arrived at ``step - max_lag`` too. Ranks that meet in
  collectives run in lockstep, so the default lag is 0 and the call is a host-side
  barrier whose failure names the missing rank. It polls with a growing sleep.
* A peer whose counter stops advancing for ``timeout_s`` (measured on this host's
  monotonic clock from the last time its value changed; set it above the longest step)
  raises ``PeerLostError``.
* ``leave(reason)`` instead of arriving at the next step: records the steps this rank
  took part in and why it leaves. Peers then raise ``PeerLostError`` with that reason
  at the first step it will miss, without waiting for the timeout.

The reference has no liveness detection: it barriers before ``destroy_process_group``
(src/utils.py:10-14) and relies on NCCL's own errors.
"""
from __future__ import annotations

import time

import torch.distributed as dist


class PeerLostError(RuntimeError):
    def __init__(self, rank: int, step: int, reason: str):
        super().__init__(f"rank {rank} is gone before step {step}: {reason}")
        self.rank, self.step, self.reason = rank, step, reason


class Heartbeat:
    def __init__(self, store, rank: int, world: int, timeout_s: float = 60.0, max_lag: int = 0,
                 prefix: str = "sepx/heartbeat"):
        if timeout_s <= 0 or max_lag < 0:
            raise ValueError("timeout_s must be > 0 and max_lag >= 0")
        self.store = dist.PrefixStore(prefix, store)
        self.rank, self.world = int(rank), int(world)
        self.timeout_s, self.max_lag = float(timeout_s), int(max_lag)
        self.arrived = 0  # steps this rank has arrived at
        self.store.add(f"count/{self.rank}", 0)  # create this rank's key
        # per peer: last count seen and when it last changed (this host's clock)
        now = time.monotonic()
        self._seen = {r: (-1, now) for r in range(self.world) if r != self.rank}

    @classmethod
    def from_default_group(cls, timeout_s: float = 60.0, max_lag: int = 0) -> "Heartbeat":
        """Heartbeat over the default process group's store."""
        from torch.distributed.distributed_c10d import _get_default_store

        return cls(_get_default_store(), dist.get_rank(), dist.get_world_size(), timeout_s, max_lag)

    def beat(self) -> int:
        """Announce arrival at the next step; returns the steps arrived at."""
        self.arrived = int(self.store.add(f"count/{self.rank}", 1))
        return self.arrived

    def arrive(self, step: int, poll_s: float = 0.001) -> None:
        """``beat()`` then ``wait(step)``: call at the start of step ``step``."""
        if self.arrived != step:
            raise ValueError(f"arrive({step}) after arriving at {self.arrived} steps: call it once per step")
        self.beat()
        self.wait(step, poll_s)

    def leave(self, reason: str = "left") -> None:
        """Leave between steps: peers learn that this rank took part in ``self.arrived``
        steps and raise at the next one."""
        self.store.set(f"left/{self.rank}", f"{self.arrived}:{reason}")

    def _left(self, r: int):
        """(steps taken part in, reason) of a peer that left, else None."""
        key = f"left/{r}"
        if self.store.check([key]):
            done, _, reason = self.store.get(key).decode(errors="replace").partition(":")
            return int(done), reason
        return None

    def wait(self, step: int, poll_s: float = 0.001) -> None:
        """Return once every peer has arrived at ``step - max_lag``; raise
        ``PeerLostError`` for a peer that left before it or stopped advancing for
        ``timeout_s``."""
        need = step + 1 - self.max_lag  # arrivals that cover step - max_lag
        pending = set(self._seen)
        sleep = poll_s
        while True:
            now = time.monotonic()
            for r in sorted(pending):
                v = int(self.store.add(f"count/{r}", 0))
                last, since = self._seen[r]
                if v != last:
                    self._seen[r] = (v, now)
                    since = now
                if v >= need:
                    pending.discard(r)
                    continue
                left = self._left(r)
                if left is not None and left[0] < need:
                    raise PeerLostError(r, step, f"left after step {left[0] - 1} ({left[1]})")
                if now - since > self.timeout_s:
                    raise PeerLostError(r, step, f"no heartbeat for {now - since:.1f} s (last arrived at step "
                                                 f"{v - 1}, step {need - 1} needed)")
            if not pending:
                return
            time.sleep(sleep)
            sleep = min(sleep * 2, 0.05)
