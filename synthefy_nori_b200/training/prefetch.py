"""Background batch generation in worker processes (reference ``training/prefetch.py:25-205``).

``DataPrefetcher(make_batch, num_workers)`` runs ``make_batch(seed)`` for seeds
``base_seed + i`` (i = 0, 1, 2, ...) in spawned worker processes and hands the results back
strictly in seed order (FIFO reassembly by sequence number), so a run is reproducible
regardless of which worker finished first.  A worker exception comes back as an error
sentinel and is re-raised in the consumer with the worker's traceback; a worker that dies
without reporting is detected by a bounded wait (``timeout_s``) and the liveness check, and
raises ``RuntimeError`` instead of blocking forever.  The GPU SCM-prior path
(``training/prior.py``) generates batches on the device and needs no prefetcher; this one
serves host-side generators.
"""

from __future__ import annotations

import multiprocessing as mp
import queue
import time
import traceback


def _worker(make_batch, tasks, results):
    while True:
        item = tasks.get()
        if item is None:
            return
        seq, seed = item
        try:
            results.put((seq, True, make_batch(seed)))
        except BaseException:  # noqa: BLE001 - forwarded to the consumer
            results.put((seq, False, traceback.format_exc()))


class DataPrefetcher:
    def __init__(self, make_batch, num_workers: int = 2, base_seed: int = 0, depth: int = 4,
                 timeout_s: float = 600.0, start_method: str = "spawn"):
        if num_workers < 1:
            raise ValueError("num_workers must be >= 1")
        ctx = mp.get_context(start_method)
        self.tasks, self.results = ctx.Queue(), ctx.Queue()
        self.workers = [ctx.Process(target=_worker, args=(make_batch, self.tasks, self.results), daemon=True)
                        for _ in range(num_workers)]
        for w in self.workers:
            w.start()
        self.base_seed, self.timeout_s = int(base_seed), float(timeout_s)
        self.next_submit = self.next_yield = 0
        self.pending: dict = {}
        for _ in range(max(depth, num_workers)):
            self._submit()

    def _submit(self) -> None:
        self.tasks.put((self.next_submit, self.base_seed + self.next_submit))
        self.next_submit += 1

    def __iter__(self):
        return self

    def __next__(self):
        deadline = time.monotonic() + self.timeout_s
        while self.next_yield not in self.pending:
            try:
                seq, ok, payload = self.results.get(timeout=0.5)
                self.pending[seq] = (ok, payload)
            except queue.Empty:
                dead = [w.pid for w in self.workers if not w.is_alive()]
                if dead:
                    self.close()
                    raise RuntimeError(f"prefetch worker(s) {dead} exited without returning batch {self.next_yield}")
                if time.monotonic() > deadline:
                    self.close()
                    raise RuntimeError(f"no batch within {self.timeout_s:.0f} s (sequence {self.next_yield})")
        ok, payload = self.pending.pop(self.next_yield)
        if not ok:
            self.close()
            raise RuntimeError(f"prefetch worker failed on batch {self.next_yield}:\n{payload}")
        self.next_yield += 1
        self._submit()
        return payload

    def state(self) -> dict:
        """Position for checkpoint/resume: the next batch's sequence number."""
        return {"base_seed": self.base_seed, "next": self.next_yield}

    def close(self) -> None:
        for _ in self.workers:
            try:
                self.tasks.put_nowait(None)
            except Exception:  # noqa: BLE001
                pass
        for w in self.workers:
            w.join(timeout=2)
            if w.is_alive():
                w.terminate()
                w.join(timeout=2)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
