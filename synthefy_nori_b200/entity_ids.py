"""Integer codes for declared identifier columns (store id, customer id, ...).

Behaviour (parity with the reference's ``entity_ids.py``): every declared column may hold
strings or integers plus missing values; ``fit`` records the distinct context values in
order of first appearance, and ``transform`` replaces each value by its position in that
list, with missing values and values never seen in the context mapped to -1.

Implementation: the context values are factorized once (``pandas.factorize`` keeps
first-appearance order); a transform is one categorical lookup per column, so it is a
vectorised hash join rather than a per-value loop.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import pandas as pd


def _id_kind(values: pd.Series) -> str | None:
    """'str', 'int', None (all missing) or 'mixed' for the non-missing values of a column."""
    present = values.dropna()
    if present.empty:
        return None
    if pd.api.types.is_bool_dtype(present):
        return "mixed"
    if pd.api.types.is_integer_dtype(present):
        return "int"
    kinds = {"str" if isinstance(v, str) else
             "int" if isinstance(v, (int, np.integer)) and not isinstance(v, (bool, np.bool_)) else "mixed"
             for v in present}
    return kinds.pop() if len(kinds) == 1 else "mixed"


@dataclass
class EntityIDPreprocessor:
    encode_id_cols: list
    categories_: dict = field(default_factory=dict, init=False)

    def __post_init__(self):
        cols = self.encode_id_cols
        if not isinstance(cols, list) or any(not isinstance(c, str) or c == "" for c in cols):
            raise ValueError("encode_id_cols: expected a list of non-empty column names")
        if len(cols) != len(set(cols)):
            raise ValueError("encode_id_cols: duplicate column name")
        self.encode_id_cols = list(cols)

    def _validated(self, X) -> pd.DataFrame:
        if not isinstance(X, pd.DataFrame) or X.columns.has_duplicates:
            raise ValueError("ID encoding needs a pandas DataFrame whose column names are unique")
        missing = [c for c in self.encode_id_cols if c not in X.columns]
        if missing:
            raise ValueError(f"ID column(s) not in the frame: {missing}")
        bad = [c for c in self.encode_id_cols if _id_kind(X[c]) == "mixed"]
        if bad:
            raise ValueError(f"ID column(s) {bad}: values must be all integers or all strings (plus missing)")
        return X

    def fit(self, X):
        X = self._validated(X)
        self.categories_ = {c: pd.Index(pd.factorize(X[c], use_na_sentinel=True)[1]) for c in self.encode_id_cols}
        return self

    def transform(self, X):
        X = self._validated(X)
        out = X.copy()
        for c, cats in self.categories_.items():
            codes = pd.Categorical(X[c], categories=cats).codes  # unseen and missing -> -1
            out[c] = codes.astype(np.int64)
        return out

    def fit_transform(self, X):
        return self.fit(X).transform(X)
