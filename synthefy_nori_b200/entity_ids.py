"""Context-fitted integer codes for declared identifier columns.

Parity target: reference ``src/synthefy_nori/entity_ids.py:7-45``: each declared column
(strings or integers, plus missing values) is replaced by the position of its value among
the distinct values seen in the context, in order of first appearance; missing values and
values unseen in the context become -1.
"""

from __future__ import annotations

import numpy as np
import pandas as pd


class EntityIDPreprocessor:
    def __init__(self, encode_id_cols):
        if not isinstance(encode_id_cols, list) or not all(isinstance(c, str) and c for c in encode_id_cols):
            raise ValueError("encode_id_cols must be a list of nonempty column names")
        if len(set(encode_id_cols)) != len(encode_id_cols):
            raise ValueError("encode_id_cols must not contain duplicate names")
        self.encode_id_cols = list(encode_id_cols)

    def _check(self, X) -> None:
        if not isinstance(X, pd.DataFrame) or not X.columns.is_unique:
            raise ValueError("encode_id_cols requires a DataFrame with unique column names")
        for c in self.encode_id_cols:
            if c not in X:
                raise ValueError(f"ID column not found: {c}")
            vals = X[c].dropna().tolist()
            strs = all(isinstance(v, str) for v in vals)
            ints = all(isinstance(v, (int, np.integer)) and not isinstance(v, (bool, np.bool_)) for v in vals)
            if vals and not (strs or ints):
                raise ValueError(f"ID column {c!r} must contain integers or strings, plus missing values")

    def fit(self, X):
        self._check(X)
        self.values_ = {c: pd.Index(pd.unique(X[c].dropna())) for c in self.encode_id_cols}
        return self

    def transform(self, X):
        self._check(X)
        out = X.copy()
        for c, index in self.values_.items():
            codes = index.get_indexer(X[c])
            codes[X[c].isna().to_numpy()] = -1
            out[c] = codes
        return out

    def fit_transform(self, X):
        return self.fit(X).transform(X)
