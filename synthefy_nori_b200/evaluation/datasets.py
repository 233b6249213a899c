"""Regression datasets for evaluation.

Parity target: reference ``evaluation/datasets.py:64-675``.  Sources:

- ``load_csv_dir(dir, source)``: ``<name>_train.csv`` (+ optional ``<name>_test.csv``,
  else an 80/20 split), the last column is the target - the layout the reference's
  TabArena / TALENT caches and ``--custom-reg-dir`` use;
- ``load_openml(ids_or_list_file)``: OpenML datasets by id (needs the ``openml`` package
  and network access; a pinned list file has ``name,openml_dataset_id`` rows);
- ``load_synthetic()``: an offline suite (Friedman 1-3, sparse linear, a nonlinear
  interaction table with missing values and categorical codes) for smoke evaluation.

Every entry is prepared inductively as in the reference (``_make_entry_from_df``):
categorical vocabularies are fitted on the training rows (unseen test values -> -1) and
numeric gaps are filled with the training medians, then 0.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np
import pandas as pd


@dataclass
class DatasetEntry:
    name: str
    source: str
    X_train: np.ndarray
    y_train: np.ndarray
    X_test: np.ndarray
    y_test: np.ndarray
    task_type: str = "regression"

    @property
    def n_train(self) -> int:
        return len(self.y_train)

    @property
    def n_test(self) -> int:
        return len(self.y_test)

    @property
    def n_features(self) -> int:
        return self.X_train.shape[1]

    def summary(self) -> dict:
        return {"name": self.name, "source": self.source, "n_train": self.n_train, "n_test": self.n_test,
                "n_features": self.n_features}


def prepare(X: pd.DataFrame, y, X_test: pd.DataFrame, y_test, name: str, source: str,
            max_train: int | None = None, seed: int = 42) -> DatasetEntry:
    X, X_test = X.copy(), X_test.copy()
    for c in X.select_dtypes(include=["object", "category", "string"]).columns:
        classes = pd.Index(pd.unique(X[c].dropna()))
        X[c] = classes.get_indexer(X[c]).astype(np.float64)
        X.loc[X[c] < 0, c] = np.nan
        X_test[c] = classes.get_indexer(X_test[c]).astype(np.float64)
    X = X.apply(pd.to_numeric, errors="coerce")
    X_test = X_test.apply(pd.to_numeric, errors="coerce")
    med = X.median()
    X = X.fillna(med).fillna(0.0)
    X_test = X_test.fillna(med).fillna(0.0)
    ytr = pd.to_numeric(pd.Series(y), errors="coerce").to_numpy(np.float64)
    yte = pd.to_numeric(pd.Series(y_test), errors="coerce").to_numpy(np.float64)
    keep = np.isfinite(ytr)
    Xtr, ytr = X.to_numpy(np.float32)[keep], ytr[keep]
    if max_train is not None and len(ytr) > max_train:
        idx = np.sort(np.random.default_rng(seed).choice(len(ytr), max_train, replace=False))
        Xtr, ytr = Xtr[idx], ytr[idx]
    keep_t = np.isfinite(yte)
    return DatasetEntry(name, source, Xtr, ytr, X_test.to_numpy(np.float32)[keep_t], yte[keep_t])


class DatasetRegistry:
    def __init__(self, max_train_samples: int = 50_000, random_state: int = 42):
        self.max_train_samples, self.random_state = max_train_samples, random_state
        self._d: dict[str, DatasetEntry] = {}

    @property
    def datasets(self) -> list[DatasetEntry]:
        return list(self._d.values())

    def add(self, e: DatasetEntry) -> None:
        self._d[f"{e.source}/{e.name}"] = e

    def list_datasets(self) -> list[str]:
        return list(self._d)

    def get(self, name: str) -> DatasetEntry:
        if name in self._d:
            return self._d[name]
        hits = [e for k, e in self._d.items() if e.name == name]
        if not hits:
            raise KeyError(name)
        return hits[0]

    def filter(self, source: str | None = None) -> list[DatasetEntry]:
        return [e for e in self._d.values() if source is None or e.source == source]

    def load_csv_dir(self, data_dir: str, source: str = "custom") -> int:
        from sklearn.model_selection import train_test_split

        n = 0
        for f in sorted(os.listdir(data_dir)):
            if not f.endswith("_train.csv"):
                continue
            name = f[: -len("_train.csv")]
            tr = pd.read_csv(os.path.join(data_dir, f))
            tp = os.path.join(data_dir, f"{name}_test.csv")
            if os.path.exists(tp):
                te = pd.read_csv(tp)
            else:
                tr, te = train_test_split(tr, test_size=0.2, random_state=self.random_state)
            self.add(prepare(tr.iloc[:, :-1], tr.iloc[:, -1], te.iloc[:, :-1], te.iloc[:, -1], name, source,
                             self.max_train_samples, self.random_state))
            n += 1
        return n

    def load_openml(self, ids, source: str = "openml") -> int:
        try:
            import openml
        except ImportError as exc:
            raise RuntimeError("OpenML datasets need the 'openml' package and network access; use load_csv_dir "
                               "with a local cache instead") from exc
        from sklearn.model_selection import train_test_split

        if isinstance(ids, str):
            rows = [ln.split(",") for ln in open(ids) if ln.strip() and not ln.startswith("#")]
            ids = [int(r[1]) for r in rows if len(r) > 1 and r[1].strip().isdigit()]
        n = 0
        for did in ids:
            ds = openml.datasets.get_dataset(int(did), download_data=True)
            if ds.default_target_attribute is None:
                continue
            X, y, _, _ = ds.get_data(target=ds.default_target_attribute)
            Xtr, Xte, ytr, yte = train_test_split(X, y, test_size=0.2, random_state=self.random_state)
            self.add(prepare(Xtr, ytr, Xte, yte, ds.name, source, self.max_train_samples, self.random_state))
            n += 1
        return n

    def load_synthetic(self, n: int = 1500, seed: int = 0) -> int:
        from sklearn.datasets import make_friedman1, make_friedman2, make_friedman3, make_regression
        from sklearn.model_selection import train_test_split

        rng = np.random.default_rng(seed)
        tables = {
            "friedman1": make_friedman1(n, 10, noise=0.5, random_state=seed),
            "friedman2": make_friedman2(n, noise=5.0, random_state=seed),
            "friedman3": make_friedman3(n, noise=0.05, random_state=seed),
            "sparse_linear": make_regression(n, 40, n_informative=6, noise=1.0, random_state=seed),
        }
        X = rng.standard_normal((n, 8))
        cat = rng.integers(0, 5, n)
        y = np.sin(2 * X[:, 0]) * X[:, 1] + 0.5 * cat + 0.1 * rng.standard_normal(n)
        X[rng.random(X.shape) < 0.05] = np.nan
        tables["interaction_missing_cat"] = (np.column_stack([X, cat]), y)
        for name, (X, y) in tables.items():
            Xtr, Xte, ytr, yte = train_test_split(pd.DataFrame(X), y, test_size=0.25, random_state=seed)
            self.add(prepare(Xtr, ytr, Xte, yte, name, "synthetic", self.max_train_samples, self.random_state))
        return len(tables)
