"""Host-side failure detection for multi-process runs: per-rank heartbeats in the process-group store.

Every rank runs a daemon thread that writes its wall-clock time under
``vlmrl/hb/<rank>`` in the c10d store every ``interval`` seconds.  Before a
step launches any kernel or collective, ``check()`` reads every rank's
heartbeat and raises ``RankFailure`` when one is older than ``timeout``
(or was never written after ``grace`` seconds).  A failed rank is thus
noticed on the host, between steps, before the survivors launch work that
would wait for it; the process-group timeout is the second line of defence
for a rank that dies inside a step, and the bounded device waits
(``vlmrl.ops.CollectiveTimeout``) the third.

Ranks that leave deliberately call ``stop(leaving=True)``, which writes a
tombstone so the others report a clean departure instead of a timeout.

No reference counterpart: the reference runs a single process and only
logs and ignores failures (``core/train.py:287-308``).
"""

from __future__ import annotations

import threading
import time
from typing import Dict, List, Optional

import torch.distributed as dist


class RankFailure(RuntimeError):
    def __init__(self, ranks: List[int], detail: str):
        super().__init__(f"rank(s) {ranks} failed: {detail}")
        self.ranks = ranks


_LEFT = -1.0


class Heartbeat:
    def __init__(self, store: Optional["dist.Store"] = None, rank: Optional[int] = None,
                 world: Optional[int] = None, *, interval: float = 0.5, timeout: float = 10.0, grace: float = 30.0,
                 prefix: str = "vlmrl/hb"):
        if store is None:
            from torch.distributed.distributed_c10d import _get_default_store

            store = _get_default_store()
        self.store = store
        self.rank = dist.get_rank() if rank is None else int(rank)
        self.world = dist.get_world_size() if world is None else int(world)
        self.interval, self.timeout, self.grace = float(interval), float(timeout), float(grace)
        self.prefix = prefix
        self.started = time.time()
        self._stop = threading.Event()
        self._beat()
        self._thread = threading.Thread(target=self._run, name=f"vlmrl-heartbeat-{self.rank}", daemon=True)
        self._thread.start()

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def _beat(self, value: Optional[float] = None) -> None:
        self.store.set(self._key(self.rank), repr(time.time() if value is None else value))

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self._beat()
            except Exception:  # the store is gone: the job is ending
                return

    def stop(self, leaving: bool = False) -> None:
        """Stop beating; ``leaving`` records a clean departure for the other ranks."""
        self._stop.set()
        self._thread.join(timeout=5 * self.interval)
        if leaving:
            self._beat(_LEFT)

    def ages(self) -> Dict[int, float]:
        """Seconds since each rank's last heartbeat (``inf`` = never seen, ``-1`` = left cleanly)."""
        now = time.time()
        out: Dict[int, float] = {}
        for r in range(self.world):
            try:
                if not self.store.check([self._key(r)]):
                    out[r] = float("inf")
                    continue
                v = float(self.store.get(self._key(r)).decode())
            except Exception:
                out[r] = float("inf")
                continue
            out[r] = -1.0 if v == _LEFT else now - v
        return out

    def check(self) -> None:
        """Raise ``RankFailure`` if any other rank is silent for longer than ``timeout`` (or has left)."""
        ages = self.ages()
        left = [r for r, a in ages.items() if a == -1.0 and r != self.rank]
        if left:
            raise RankFailure(left, "left the job")
        in_grace = time.time() - self.started < self.grace
        dead = [r for r, a in ages.items() if r != self.rank and a > self.timeout and not (a == float("inf") and in_grace)]
        if dead:
            raise RankFailure(dead, f"no heartbeat for more than {self.timeout:.1f} s")


__all__ = ["Heartbeat", "RankFailure"]
