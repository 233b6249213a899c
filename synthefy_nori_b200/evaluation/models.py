"""Models for the evaluation runner (reference ``evaluation/models.py``).

``ModelRegistry`` maps labels to evaluation callables ``(X_train, y_train, X_test) ->
predictions``: Nori checkpoints or presets (optionally with an inference config, an
ensemble size or a memory policy), checkpoint families added from a directory
(``add_checkpoints("run/", prefix="step")`` registers every ``*.pt`` with its step), and
classical baselines from scikit-learn (ridge, k-nearest neighbours, random forest,
histogram gradient boosting) for context.  Nori models are loaded once per label and
reused across datasets.
"""

from __future__ import annotations

import glob
import os
import re
from dataclasses import dataclass, field
from typing import Callable

import numpy as np


@dataclass
class ModelEntry:
    label: str
    kind: str  # "nori" | "baseline"
    kwargs: dict = field(default_factory=dict)


def _baseline(name: str, seed: int = 0):
    from sklearn.ensemble import HistGradientBoostingRegressor, RandomForestRegressor
    from sklearn.impute import SimpleImputer
    from sklearn.linear_model import RidgeCV
    from sklearn.neighbors import KNeighborsRegressor
    from sklearn.pipeline import make_pipeline
    from sklearn.preprocessing import StandardScaler

    if name == "ridge":
        return make_pipeline(SimpleImputer(), StandardScaler(), RidgeCV(alphas=np.logspace(-3, 3, 13)))
    if name == "knn":
        return make_pipeline(SimpleImputer(), StandardScaler(), KNeighborsRegressor(n_neighbors=10))
    if name == "random_forest":
        return make_pipeline(SimpleImputer(), RandomForestRegressor(n_estimators=300, n_jobs=-1, random_state=seed))
    if name == "hist_gbdt":
        return HistGradientBoostingRegressor(random_state=seed)
    raise ValueError(f"unknown baseline {name!r}")


BASELINES = ("ridge", "knn", "random_forest", "hist_gbdt")


class ModelRegistry:
    def __init__(self, device=None):
        self.device = device
        self.entries: dict[str, ModelEntry] = {}
        self._loaded: dict[str, object] = {}

    def register(self, entry: ModelEntry) -> None:
        if entry.label in self.entries:
            raise ValueError(f"model label {entry.label!r} already registered")
        self.entries[entry.label] = entry

    def add_nori(self, label: str, *, model_path: str | None = None, model: str | None = None, weights=None,
                 **regressor_kwargs) -> None:
        self.register(ModelEntry(label, "nori", dict(model_path=model_path, model=model, weights=weights,
                                                     **regressor_kwargs)))

    def add_checkpoints(self, directory: str, prefix: str = "ckpt", pattern: str = "*.pt", **kw) -> list[str]:
        """Register every checkpoint of a run directory as ``<prefix>-<step>`` (step from
        the file name, else its order)."""
        files = sorted(glob.glob(os.path.join(directory, pattern)))
        labels = []
        for i, f in enumerate(files):
            nums = re.findall(r"(\d+)", os.path.basename(f))
            label = f"{prefix}-{nums[-1] if nums else i}"
            self.add_nori(label, model_path=f, **kw)
            labels.append(label)
        return labels

    def add_baselines(self, names=BASELINES, seed: int = 0) -> None:
        for n in names:
            self.register(ModelEntry(n, "baseline", {"seed": seed}))

    def list_models(self) -> list[str]:
        return list(self.entries)

    def get(self, label: str) -> Callable:
        e = self.entries[label]
        if e.kind == "baseline":
            def fn(Xtr, ytr, Xte, name=label, seed=e.kwargs.get("seed", 0)):
                return _baseline(name, seed).fit(Xtr, ytr).predict(Xte)

            return fn
        from synthefy_nori_b200.api import NoriRegressor

        def fn(Xtr, ytr, Xte, e=e):
            reg = NoriRegressor(device=self.device, **{k: v for k, v in e.kwargs.items() if v is not None})
            if label in self._loaded:
                reg._model_obj = self._loaded[label]
            out = reg.fit(Xtr, ytr).predict(Xte)
            self._loaded[label] = reg._load_model()
            return out

        return fn

    def callables(self) -> dict[str, Callable]:
        return {label: self.get(label) for label in self.entries}

    def cleanup(self) -> None:
        self._loaded.clear()
        try:
            import torch

            if torch.cuda.is_available():
                torch.cuda.empty_cache()
        except ImportError:
            pass


def benchmark_list(name: str) -> str:
    """Path of a pinned benchmark list shipped with the package (``tabarena_reg``,
    ``talent_reg``)."""
    path = os.path.join(os.path.dirname(__file__), "benchmark_lists", f"{name}.csv")
    if not os.path.isfile(path):
        raise FileNotFoundError(f"no pinned benchmark list {name!r}")
    return path
