"""Host-side failure detection for the multi-rank paths (one process per GPU).

The reference engine is a single process. Its failure handling is a step error sent to every
active sequence (engine/crates/engine/src/scheduler.rs:210-216). Across ranks, the others must
notice a rank that crashed or left before they launch work that waits for it: an NCCL
collective, or the head-sharded NVLink gather (whose bounded device wait would report
LT_E_TIMEOUT only after 2 s).

``RankHealth`` keeps one heartbeat per rank in the torch.distributed store:
  - ``beat(step)`` publishes this rank's step counter;
  - ``check(step)`` waits, bounded by ``timeout_s``, until every peer has published at least
    ``step``. It raises ``PeerLost`` naming the ranks that announced they left (``leave()``)
    or that stayed silent;
  - ``leave()`` marks this rank as gone, so the others learn it at once instead of after the
    timeout.

Calls go between steps, never around a launch in flight. A rank that leaves does so with none
of its kernels or collectives outstanding.
"""
from __future__ import annotations

import time


class PeerLost(RuntimeError):
    """Raised by RankHealth.check: the ranks in ``ranks`` left or fell silent."""

    def __init__(self, ranks, step: int, reason: str):
        super().__init__(f"rank(s) {sorted(ranks)} {reason} before step {step}")
        self.ranks = sorted(ranks)
        self.step = step
        self.reason = reason


class RankHealth:
    def __init__(self, store, rank: int, world: int, *, prefix: str = "lt_health", timeout_s: float = 2.0,
                 poll_s: float = 0.002):
        self.store, self.rank, self.world = store, rank, world
        self.prefix, self.timeout_s, self.poll_s = prefix, timeout_s, poll_s

    def _beat_key(self, r: int) -> str:
        return f"{self.prefix}/beat/{r}"

    def _left_key(self, r: int) -> str:
        return f"{self.prefix}/left/{r}"

    def beat(self, step: int) -> None:
        self.store.set(self._beat_key(self.rank), str(int(step)))

    def leave(self) -> None:
        self.store.set(self._left_key(self.rank), "1")

    def check(self, step: int) -> None:
        """Every peer has reached ``step``, or PeerLost within timeout_s."""
        pending = {r for r in range(self.world) if r != self.rank}
        deadline = time.monotonic() + self.timeout_s
        while pending:
            left = {r for r in pending if self.store.check([self._left_key(r)])}
            if left:
                raise PeerLost(left, step, "left")
            for r in list(pending):
                key = self._beat_key(r)
                if self.store.check([key]) and int(self.store.get(key)) >= step:
                    pending.discard(r)
            if pending:
                if time.monotonic() > deadline:
                    raise PeerLost(pending, step, f"sent no heartbeat within {self.timeout_s:g} s")
                time.sleep(self.poll_s)
