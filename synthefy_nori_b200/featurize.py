"""DataFrame -> numeric matrix, fitted once on the context rows.

Parity target: reference ``libs/synthefy/src/synthefy/featurize.py:102-486``
(``DataFramePreprocessor``) and ``text_features.py`` (text columns -> sentence
embedding -> TruncatedSVD).  Column roles are resolved at ``fit``: numeric columns pass
through; categorical columns (``categorical_columns="auto"`` = every non-numeric,
non-text column, or an explicit list) become ordinal codes over their sorted training
levels (explicit columns above ``max_categorical_cardinality`` keep the most frequent K
levels, rarer and unseen values share one "other" code; missing stays NaN) or one-hot
groups; text columns become dense vectors reduced by TruncatedSVD.  ``transform``
replays the fitted schema and never learns from query rows.

Text embedding: the reference encodes text with a sentence-transformer model
(``embedder="minilm"``), which needs a model download.  This build ships a
self-contained ``embedder="hashing"`` (signed feature hashing of word and character
3-gram counts, L2-normalised) and accepts any callable ``list[str] -> ndarray``; the
sentence-transformer path is used when that package and its weights are present.
"""

from __future__ import annotations

import hashlib
from collections import Counter
from typing import Any

import numpy as np
import pandas as pd

CATEGORICAL_ENCODINGS = ("ordinal", "onehot")


def _is_numeric(s: pd.Series) -> bool:
    return not isinstance(s.dtype, pd.CategoricalDtype) and pd.api.types.is_numeric_dtype(s)


def _is_temporal(s: pd.Series) -> bool:
    return (pd.api.types.is_datetime64_any_dtype(s) or pd.api.types.is_timedelta64_dtype(s)
            or isinstance(s.dtype, pd.PeriodDtype))


def _key(v: Any) -> str:
    if isinstance(v, np.generic):
        v = v.item()
    if isinstance(v, float) and v.is_integer():
        v = int(v)
    return str(v)


def _columns(value, name: str, allow_auto: bool = False) -> tuple[str | None, list]:
    if value is None:
        return None, []
    if isinstance(value, str):
        if allow_auto and value == "auto":
            return "auto", []
        return None, [value]
    try:
        cols = list(value)
    except TypeError as exc:
        raise TypeError(f"{name} must be a column name, a sequence of names or None") from exc
    if len(set(map(repr, cols))) != len(cols):
        raise ValueError(f"{name} contains duplicate names")
    return None, cols


def hashing_embedder(texts: list[str], dim: int = 512) -> np.ndarray:
    """Signed feature hashing of lower-cased word unigrams and character 3-grams."""
    out = np.zeros((len(texts), dim), dtype=np.float32)
    for i, t in enumerate(texts):
        t = "" if t is None else str(t).lower()
        grams = t.split() + [t[j : j + 3] for j in range(max(len(t) - 2, 0))]
        for g in grams:
            h = int.from_bytes(hashlib.blake2b(g.encode(), digest_size=8).digest(), "little")
            out[i, h % dim] += 1.0 if (h >> 63) & 1 else -1.0
        n = np.linalg.norm(out[i])
        if n > 0:
            out[i] /= n
    return out


class TextFeaturizer:
    """Text columns -> one embedding per cell -> TruncatedSVD to ``svd_dim`` per column."""

    def __init__(self, columns: list, *, svd_dim: int | None = 128, embedder: Any = "hashing"):
        self.columns, self.svd_dim, self.embedder = list(columns), svd_dim, embedder

    def _embed(self, texts: list[str]) -> np.ndarray:
        if callable(self.embedder):
            return np.asarray(self.embedder(texts), dtype=np.float32)
        if self.embedder == "hashing":
            return hashing_embedder(texts)
        try:
            from sentence_transformers import SentenceTransformer
        except ImportError as exc:
            raise RuntimeError(f"embedder={self.embedder!r} needs sentence-transformers; use embedder='hashing' or a "
                               "callable") from exc
        name = "sentence-transformers/all-MiniLM-L6-v2" if self.embedder == "minilm" else self.embedder
        return np.asarray(SentenceTransformer(name).encode(texts), dtype=np.float32)

    def fit_transform(self, frame: pd.DataFrame) -> np.ndarray:
        from sklearn.decomposition import TruncatedSVD

        self.svds_, blocks = {}, []
        for c in self.columns:
            e = self._embed(frame[c].astype(object).where(frame[c].notna(), "").astype(str).tolist())
            k = e.shape[1] if self.svd_dim is None else min(self.svd_dim, e.shape[1] - 1, max(e.shape[0] - 1, 1))
            if self.svd_dim is not None and k >= 1:
                svd = TruncatedSVD(n_components=k, random_state=0).fit(e)
                self.svds_[c] = svd
                e = svd.transform(e)
            blocks.append(e.astype(np.float32))
        return np.hstack(blocks)

    def transform(self, frame: pd.DataFrame) -> np.ndarray:
        blocks = []
        for c in self.columns:
            e = self._embed(frame[c].astype(object).where(frame[c].notna(), "").astype(str).tolist())
            if c in self.svds_:
                e = self.svds_[c].transform(e)
            blocks.append(e.astype(np.float32))
        return np.hstack(blocks)


class DataFramePreprocessor:
    def __init__(self, *, categorical_columns: Any = "auto", text_columns: Any = None,
                 max_categorical_cardinality: int = 100, categorical_encoding: str = "ordinal",
                 svd_dim: int | None = 128, embedder: Any = "hashing"):
        self.categorical_columns = categorical_columns
        self.text_columns = text_columns
        self.max_categorical_cardinality = max_categorical_cardinality
        self.categorical_encoding = categorical_encoding
        self.svd_dim = svd_dim
        self.embedder = embedder

    @staticmethod
    def _frame(X, name: str = "X") -> pd.DataFrame:
        if not isinstance(X, pd.DataFrame):
            raise TypeError(f"{name} must be a pandas DataFrame; got {type(X).__name__}")
        if not X.columns.is_unique:
            raise ValueError(f"{name} has duplicate column names")
        if X.shape[1] == 0:
            raise ValueError(f"{name} must contain at least one feature column")
        return X

    def fit_transform(self, X) -> pd.DataFrame:
        X = self._frame(X)
        if not isinstance(self.max_categorical_cardinality, int) or self.max_categorical_cardinality < 1:
            raise ValueError("max_categorical_cardinality must be a positive integer")
        if self.categorical_encoding not in CATEGORICAL_ENCODINGS:
            raise ValueError(f"categorical_encoding must be one of {CATEGORICAL_ENCODINGS}")
        mode, declared_cat = _columns(self.categorical_columns, "categorical_columns", allow_auto=True)
        _, declared_text = _columns(self.text_columns, "text_columns")
        for name, cols in (("categorical_columns", declared_cat), ("text_columns", declared_text)):
            missing = [c for c in cols if c not in X.columns]
            if missing:
                raise ValueError(f"{name} not found in the DataFrame: {missing}")
        if set(declared_cat) & set(declared_text):
            raise ValueError("categorical_columns and text_columns must not overlap")
        numeric, categorical, temporal, undeclared = [], [], [], []
        for c in X.columns:
            if c in declared_text:
                continue
            s = X[c]
            if _is_temporal(s):
                temporal.append(c)
            elif c in declared_cat:
                categorical.append(c)
            elif _is_numeric(s):
                numeric.append(c)
            elif mode == "auto":
                categorical.append(c)
            else:
                undeclared.append(c)
        if temporal:
            raise ValueError(f"temporal feature columns are not inferred: {temporal}; convert them to numbers or strings")
        if undeclared:
            raise ValueError(f"non-numeric feature columns have no declared role: {undeclared}")
        self.columns_ = list(X.columns)
        self.n_features_in_ = len(self.columns_)
        self.numeric_columns_, self.categorical_columns_, self.text_columns_ = numeric, categorical, declared_text
        explicit = set(declared_cat) | {c for c in categorical if isinstance(X[c].dtype, pd.CategoricalDtype)}
        self.category_maps_, self.category_has_missing_ = {}, {}
        K = self.max_categorical_cardinality
        for c in categorical:
            s = X[c]
            counts = Counter(_key(v) for v in s[s.notna()].tolist())
            if len(counts) > K and c not in explicit:
                raise ValueError(f"column {c!r} has {len(counts)} distinct values (> max_categorical_cardinality={K}); "
                                 "declare it in categorical_columns or text_columns")
            keep = sorted(counts, key=lambda k: (-counts[k], k))[:K] if len(counts) > K else list(counts)
            self.category_maps_[c] = {k: i for i, k in enumerate(sorted(keep))}
            self.category_has_missing_[c] = bool(s.isna().any())
        self._text = None
        text = None
        if declared_text:
            self._text = TextFeaturizer(declared_text, svd_dim=self.svd_dim, embedder=self.embedder)
            text = self._text.fit_transform(X)
        out = self._assemble(X, text)
        self.feature_names_out_ = np.asarray(out.columns, dtype=object)
        self.n_features_out_ = out.shape[1]
        return out

    def fit(self, X, y=None):
        self.fit_transform(X)
        return self

    def transform(self, X) -> pd.DataFrame:
        if not hasattr(self, "columns_"):
            raise RuntimeError("call fit() before transform()")
        X = self._frame(X)
        missing = [c for c in self.columns_ if c not in X.columns]
        extra = [c for c in X.columns if c not in self.columns_]
        if missing or extra:
            raise ValueError(f"query schema does not match the fitted schema: missing={missing}, extra={extra}")
        X = X.loc[:, self.columns_]
        bad = [c for c in self.numeric_columns_ if not _is_numeric(X[c])]
        if bad:
            raise ValueError(f"fitted numeric columns are not numeric in the query: {bad}")
        text = self._text.transform(X) if self._text is not None else None
        out = self._assemble(X, text)
        if list(out.columns) != list(self.feature_names_out_):
            raise RuntimeError("DataFrame preprocessing produced a different feature layout at transform time")
        return out

    def _assemble(self, X: pd.DataFrame, text) -> pd.DataFrame:
        blocks, names = [], []
        for c in self.columns_:
            if c in self.numeric_columns_:
                blocks.append(pd.to_numeric(X[c]).to_numpy(np.float32).reshape(-1, 1))
                names.append(c)
            elif c in self.category_maps_:
                mp = self.category_maps_[c]
                other = len(mp)
                s = X[c]
                na = s.isna().to_numpy()
                codes = np.array([np.nan if m else mp.get(_key(v), other) for v, m in zip(s.tolist(), na)],
                                 dtype=np.float32)
                if self.categorical_encoding == "ordinal":
                    blocks.append(codes.reshape(-1, 1))
                    names.append(c)
                else:
                    has_na = self.category_has_missing_[c]
                    oh = np.zeros((len(s), len(mp) + int(has_na)), dtype=np.float32)
                    valid = ~np.isnan(codes) & (np.nan_to_num(codes, nan=other) < other)
                    oh[np.flatnonzero(valid), codes[valid].astype(np.int64)] = 1.0
                    if has_na:
                        oh[na, len(mp)] = 1.0
                    blocks.append(oh)
                    names += [f"{c}_{k}" for k in sorted(mp, key=mp.get)] + ([f"{c}_nan"] if has_na else [])
        if text is not None:
            blocks.append(np.asarray(text, dtype=np.float32))
            names += [f"text__{i}" for i in range(text.shape[1])]
        if not blocks:
            raise ValueError("no usable feature columns remain after DataFrame preprocessing")
        if len(set(map(str, names))) != len(names):
            raise ValueError("generated column names collide; rename the input columns")
        return pd.DataFrame(np.hstack(blocks), index=X.index, columns=names)

    def get_feature_names_out(self, input_features=None) -> np.ndarray:
        return self.feature_names_out_.copy()


def align_and_featurize(X_train, X_test, **kw):
    """Fit a ``DataFramePreprocessor`` on ``X_train`` and apply it to both frames."""
    pre = DataFramePreprocessor(**kw)
    return pre.fit_transform(X_train), pre.transform(X_test), pre
