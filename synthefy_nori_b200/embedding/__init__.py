"""Nori embeddings as a scikit-learn transformer, with out-of-fold training embeddings.

Parity target: reference ``src/synthefy_nori/embedding/embedding.py:13-155``
(``NoriEmbedding(n_fold, model=..., shuffle, random_state)``; ``fit`` stores
``train_embeddings_`` and refits on the whole training set; ``transform`` always embeds
through the full-data model; output ``[members, rows, embed_dim]``).

A row's out-of-fold embedding comes from a context that does not contain it: the
training rows are split into ``n_fold`` folds (scikit-learn's ``KFold``, so a given
``random_state`` makes the same split as the reference) and each fold is embedded as
query rows against the other folds as context.  The estimator is fitted once per fold
on the same ``NoriRegressor`` instance: ``fit`` only replaces the context arrays, so the
loaded checkpoint, its persistent bf16 weight layouts and the device predictor are
built once and shared by every fold and by the final full-data fit.
"""

from __future__ import annotations

import numpy as np
from sklearn.base import BaseEstimator, TransformerMixin, clone
from sklearn.model_selection import KFold
from sklearn.utils.validation import check_is_fitted


class NoriEmbedding(TransformerMixin, BaseEstimator):
    """``n_fold=0``: one fit on all rows embeds both training and new rows.
    ``n_fold>=2``: ``train_embeddings_`` are out-of-fold (row order preserved); ``model_``
    is then refitted on every row for ``transform``.  ``model`` (a ``NoriRegressor``) is
    required and is cloned, never modified."""

    def __init__(self, n_fold: int = 0, *, model=None, shuffle: bool = False, random_state: int | None = None):
        self.n_fold = n_fold
        self.model = model
        self.shuffle = shuffle
        self.random_state = random_state

    def _template(self):
        if self.model is None:
            raise ValueError("NoriEmbedding needs model=NoriRegressor(model=<a preset or checkpoint>); "
                             "no default model is chosen on the caller's behalf")
        return clone(self.model)

    def _out_of_fold(self, X: np.ndarray, y: np.ndarray) -> np.ndarray:
        split = KFold(n_splits=self.n_fold, shuffle=self.shuffle,
                      random_state=self.random_state if self.shuffle else None)
        out = None
        for ctx, held in split.split(X):
            self.model_.fit(X[ctx], y[ctx])
            emb = np.asarray(self.model_.get_embeddings(X[held], data_source="test"))
            if out is None:  # [members, rows, E] in the caller's row order
                out = np.empty((emb.shape[0], len(X)) + emb.shape[2:], dtype=emb.dtype)
            out[:, held] = emb
        return out

    def fit(self, X, y) -> "NoriEmbedding":
        if self.n_fold < 0 or self.n_fold == 1:
            raise ValueError("n_fold must be 0 (no folds) or at least 2")
        X, y = np.asarray(X), np.asarray(y)
        self.model_ = self._template()
        if self.n_fold == 0:
            self.model_.fit(X, y)
            self.train_embeddings_ = np.asarray(self.model_.get_embeddings(X, data_source="test"))
            return self
        if self.n_fold > len(X):
            raise ValueError(f"n_fold={self.n_fold} exceeds the {len(X)} training rows")
        self.train_embeddings_ = self._out_of_fold(X, y)
        self.model_.fit(X, y)
        return self

    def transform(self, X) -> np.ndarray:
        """Embeddings of ``X`` from the full-data model (never the cached out-of-fold ones)."""
        check_is_fitted(self, "model_")
        return np.asarray(self.model_.get_embeddings(np.asarray(X), data_source="test"))

    def fit_transform(self, X, y=None, **fit_params) -> np.ndarray:
        if y is None:
            raise ValueError("NoriEmbedding.fit_transform needs the target y (it is the context's label)")
        return self.fit(X, y).train_embeddings_


__all__ = ["NoriEmbedding"]
