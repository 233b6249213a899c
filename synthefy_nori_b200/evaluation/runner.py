"""Evaluation runner (reference ``evaluation/runner.py:45-510``).

Runs every model over every dataset with the degradation guard on
(``strict_pipeline(SvdFallbackWarning)``: a silently degraded prediction is recorded as
an error, not a score), records R^2 / RMSE / MAE, latency and throughput, caches each
(model, dataset) result as JSON keyed by a hash of the evaluation parameters, and writes
``results.csv`` plus a per-model summary.
"""

from __future__ import annotations

import hashlib
import json
import os
import time
from dataclasses import asdict, dataclass, field
from typing import Callable

import numpy as np
import pandas as pd

from synthefy_nori_b200.inference.degradation import SvdFallbackWarning, strict_pipeline


def compute_reg_metrics(y_true, y_pred) -> dict:
    yt, yp = np.asarray(y_true, np.float64), np.asarray(y_pred, np.float64)
    ok = np.isfinite(yt) & np.isfinite(yp)
    yt, yp = yt[ok], yp[ok]
    if len(yt) < 2:
        return {"r2": float("nan"), "rmse": float("nan"), "mae": float("nan")}
    ss = ((yt - yt.mean()) ** 2).sum()
    return {"r2": float(1 - ((yt - yp) ** 2).sum() / ss) if ss > 0 else float("nan"),
            "rmse": float(np.sqrt(((yt - yp) ** 2).mean())), "mae": float(np.abs(yt - yp).mean())}


@dataclass
class EvalResult:
    model: str
    dataset: str
    source: str
    task_type: str = "regression"
    n_train: int = 0
    n_test: int = 0
    n_features: int = 0
    latency_ms: float = 0.0
    throughput_sps: float = 0.0
    error: str | None = None
    metrics: dict = field(default_factory=dict)

    def to_dict(self) -> dict:
        d = asdict(self)
        d.update(d.pop("metrics"))
        return d


class EvalRunner:
    """``models``: name -> callable ``(X_train, y_train, X_test) -> predictions``."""

    def __init__(self, models: dict[str, Callable], datasets, output_dir: str = "results/eval", warmup_runs: int = 0,
                 skip_on_error: bool = True, cache_dir: str | None = None, no_cache: bool = False,
                 max_samples: int = 50_000, verbose: bool = True):
        self.models, self.datasets = models, datasets
        self.output_dir = output_dir
        os.makedirs(output_dir, exist_ok=True)
        self.warmup_runs, self.skip_on_error, self.verbose = warmup_runs, skip_on_error, verbose
        self.cache_dir = None if no_cache else (cache_dir or os.path.join(output_dir, "cache"))
        if self.cache_dir:
            os.makedirs(self.cache_dir, exist_ok=True)
        self.max_samples = max_samples
        self.results: list[EvalResult] = []
        self.cache_hits = 0

    def _key(self, model: str, e) -> str:
        raw = f"{model}|{e.name}|{e.source}|{e.task_type}|max={self.max_samples}"
        return hashlib.sha256(raw.encode()).hexdigest()[:16]

    def evaluate_one(self, name: str, fn: Callable, e) -> EvalResult:
        path = os.path.join(self.cache_dir, self._key(name, e) + ".json") if self.cache_dir else None
        if path and os.path.exists(path):
            d = json.load(open(path))
            metrics = {k: d.pop(k) for k in ("r2", "rmse", "mae") if k in d}
            self.cache_hits += 1
            return EvalResult(**{k: v for k, v in d.items() if k in EvalResult.__dataclass_fields__}, metrics=metrics)
        r = EvalResult(name, e.name, e.source, e.task_type, e.n_train, e.n_test, e.n_features)
        try:
            with strict_pipeline(SvdFallbackWarning):
                for _ in range(self.warmup_runs):
                    fn(e.X_train, e.y_train, e.X_test[: min(16, e.n_test)])
                t0 = time.perf_counter()
                pred = np.asarray(fn(e.X_train, e.y_train, e.X_test), np.float64).reshape(-1)
                dt = time.perf_counter() - t0
            r.latency_ms = dt * 1e3
            r.throughput_sps = e.n_test / dt if dt > 0 else 0.0
            r.metrics = compute_reg_metrics(e.y_test, pred)
        except Exception as exc:  # noqa: BLE001
            if not self.skip_on_error:
                raise
            r.error = f"{type(exc).__name__}: {exc}"
        if path and r.error is None:
            json.dump(r.to_dict(), open(path, "w"))
        return r

    def run(self) -> pd.DataFrame:
        for e in self.datasets:
            for name, fn in self.models.items():
                r = self.evaluate_one(name, fn, e)
                self.results.append(r)
                if self.verbose:
                    msg = r.error or f"r2={r.metrics.get('r2', float('nan')):.4f} {r.latency_ms:.0f} ms"
                    print(f"[{name}] {e.source}/{e.name}: {msg}", flush=True)
        df = pd.DataFrame([r.to_dict() for r in self.results])
        df.to_csv(os.path.join(self.output_dir, "results.csv"), index=False)
        self.summary(df).to_csv(os.path.join(self.output_dir, "summary.csv"))
        return df

    @staticmethod
    def summary(df: pd.DataFrame) -> pd.DataFrame:
        ok = df[df["error"].isna()] if "error" in df else df
        if ok.empty:
            return pd.DataFrame()
        return ok.groupby("model").agg(mean_r2=("r2", "mean"), median_r2=("r2", "median"), mean_rmse=("rmse", "mean"),
                                       n=("r2", "size"), total_latency_s=("latency_ms", lambda s: s.sum() / 1e3))


def nori_model_fn(**regressor_kwargs) -> Callable:
    """Evaluation callable around ``NoriRegressor`` (one fit + predict per dataset)."""
    from synthefy_nori_b200.api import NoriRegressor

    def fn(Xtr, ytr, Xte):
        return NoriRegressor(**regressor_kwargs).fit(Xtr, ytr).predict(Xte)

    return fn
