"""Host-side rank liveness for multi-process jobs.

Every rank writes a heartbeat ``"<step> <unix time>"`` into the process group's
key-value store before it launches a step, and a rank that leaves cleanly writes
``"left"``.  ``check()`` runs on every rank before the next launch and raises
``RankFailure`` (naming the ranks) when a peer announced that it left, or when its last
heartbeat is older than ``stale_s`` seconds or more than ``max_lag`` steps behind.  A
rank that dies without announcing it is caught by the staleness limit, and, as the last
bound, by the process group's own collective timeout.

So the survivors learn of a failure on the host, between steps, with none of their
kernels or collectives in flight (the collective timeout only fires if a rank is lost
in the middle of a step).  The reference relies on NCCL's timeout alone for DDP ranks
and on liveness polling for its prefetch workers (``training/prefetch.py``).
"""

from __future__ import annotations

import time


class RankFailure(RuntimeError):
    def __init__(self, ranks: list[int], why: str):
        super().__init__(f"rank(s) {ranks} failed: {why}")
        self.ranks = ranks
        self.why = why


class RankHealth:
    def __init__(self, store, rank: int, world: int, prefix: str = "nori/health", stale_s: float = 120.0,
                 max_lag: int = 2):
        self.store, self.rank, self.world = store, rank, world
        self.prefix, self.stale_s, self.max_lag = prefix, float(stale_s), int(max_lag)

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self, step: int) -> None:
        self.store.set(self._key(self.rank), f"{int(step)} {time.time():.3f}")

    def leave(self) -> None:
        """Announce a clean exit (call between steps, before the process ends)."""
        self.store.set(self._key(self.rank), "left")

    def status(self) -> dict:
        """``{rank: (step, age_s) | "left" | None}`` for every rank (None: never beat)."""
        now = time.time()
        out = {}
        for r in range(self.world):
            k = self._key(r)
            if not self.store.check([k]):
                out[r] = None
                continue
            v = self.store.get(k).decode()
            if v == "left":
                out[r] = "left"
            else:
                s, t = v.split()
                out[r] = (int(s), now - float(t))
        return out

    def check(self, step: int) -> None:
        """Raise ``RankFailure`` if a peer left, went stale or fell behind ``step``."""
        left, stale = [], []
        for r, st in self.status().items():
            if r == self.rank or st is None:
                continue
            if st == "left":
                left.append(r)
            elif st[1] > self.stale_s or step - st[0] > self.max_lag:
                stale.append(r)
        if left:
            raise RankFailure(left, "left the job")
        if stale:
            raise RankFailure(stale, f"no heartbeat within {self.stale_s:g} s / {self.max_lag} steps")
