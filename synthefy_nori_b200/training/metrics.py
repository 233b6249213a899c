"""Training telemetry: NVTX ranges, per-phase device timing and a metrics sink.

* ``phase(name)``: an NVTX range (visible in Nsight Systems / ncu timelines) and, when a
  ``PhaseTimer`` is active, a pair of CUDA events on the current stream, so a step can
  report forward / backward / optimizer device times without synchronising inside it.
* ``PhaseTimer.collect()`` reads the events after the caller's own synchronisation point
  (e.g. the logging interval) and, with a process group, returns the max over ranks.
* ``MetricsSink`` writes one JSON line per record to a file (and stdout on rank 0), and
  forwards to Weights & Biases when the ``wandb`` package is importable and a project is
  given (the reference logs there, ``training/trainer.py`` W&B calls).
"""

from __future__ import annotations

import contextlib
import json
import os
import time

import torch

_ACTIVE: list = []


@contextlib.contextmanager
def phase(name: str):
    cuda = torch.cuda.is_available() and torch.cuda.is_initialized()
    if cuda:
        torch.cuda.nvtx.range_push(name)
    timer = _ACTIVE[-1] if _ACTIVE else None
    ev = None
    if timer is not None and cuda:
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record()
    try:
        yield
    finally:
        if ev is not None:
            ev[1].record()
            timer.events.setdefault(name, []).append(ev)
        if cuda:
            torch.cuda.nvtx.range_pop()


class PhaseTimer:
    """Collects per-phase CUDA events while active (``with timer: ...``)."""

    def __init__(self):
        self.events: dict = {}

    def __enter__(self):
        _ACTIVE.append(self)
        return self

    def __exit__(self, *exc):
        _ACTIVE.remove(self)
        return False

    def collect(self, group=None) -> dict:
        """Milliseconds per phase (summed over its occurrences); max over ranks if a
        process group is initialised.  Synchronises on the last event."""
        names = sorted(self.events)
        out = {}
        for n in names:
            evs = self.events[n]
            evs[-1][1].synchronize()
            out[n] = sum(a.elapsed_time(b) for a, b in evs)
        import torch.distributed as dist

        if names and dist.is_available() and dist.is_initialized():
            dev = torch.device("cuda", torch.cuda.current_device())
            t = torch.tensor([out[n] for n in names], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
            out = dict(zip(names, t.tolist()))
        self.events = {}
        return {k: round(v, 3) for k, v in out.items()}


class MetricsSink:
    def __init__(self, path: str | None = None, rank: int = 0, wandb_project: str | None = None,
                 run_name: str | None = None, config: dict | None = None, echo: bool = True,
                 wandb_kwargs: dict | None = None):
        self.rank, self.echo = rank, echo
        self.f = None
        if path and rank == 0:
            os.makedirs(os.path.dirname(os.path.abspath(path)) or ".", exist_ok=True)
            self.f = open(path, "a", buffering=1)
        self.wandb = None
        if wandb_project and rank == 0:
            try:
                import wandb  # noqa: PLC0415

                self.wandb = wandb.init(project=wandb_project, name=run_name, config=config or {},
                                        **(wandb_kwargs or {}))
            except Exception:  # noqa: BLE001 - optional dependency / offline machine
                self.wandb = None

    def log(self, record: dict, step: int | None = None) -> None:
        if self.rank != 0:
            return
        rec = {"time": round(time.time(), 3), **({"step": step} if step is not None else {}), **record}
        line = json.dumps(rec, default=float)
        if self.f is not None:
            self.f.write(line + "\n")
        if self.echo:
            print(line, flush=True)
        if self.wandb is not None:
            self.wandb.log({k: v for k, v in record.items() if isinstance(v, (int, float))}, step=step)

    def close(self) -> None:
        if self.f is not None:
            self.f.close()
            self.f = None
        if self.wandb is not None:
            self.wandb.finish()
            self.wandb = None
