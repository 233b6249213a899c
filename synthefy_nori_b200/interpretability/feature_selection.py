"""Sequential feature selection (reference ``interpretability/feature_selection.py:18-100``):
scikit-learn's ``SequentialFeatureSelector`` around the (sklearn-compatible)
``NoriRegressor``, with baseline-vs-selected cross-validated scores."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np


@dataclass
class FeatureSelectionResult:
    selector: Any
    support_mask: Any
    selected_indices: list
    selected_names: list | None
    baseline_score_mean: float
    baseline_score_std: float
    selected_score_mean: float
    selected_score_std: float


def feature_selection(estimator, X, y, n_features_to_select, *, feature_names=None, cv=5, scoring=None,
                      direction: str = "forward", n_jobs=None, tol=None, **kwargs) -> FeatureSelectionResult:
    from sklearn.feature_selection import SequentialFeatureSelector
    from sklearn.model_selection import cross_val_score

    X, y = np.asarray(X), np.asarray(y)
    sfs = SequentialFeatureSelector(estimator, n_features_to_select=n_features_to_select, cv=cv, scoring=scoring,
                                    direction=direction, n_jobs=n_jobs, tol=tol, **kwargs).fit(X, y)
    mask = sfs.get_support()
    idx = [int(i) for i in np.flatnonzero(mask)]
    base = cross_val_score(estimator, X, y, cv=cv, scoring=scoring)
    sel = cross_val_score(estimator, X[:, mask], y, cv=cv, scoring=scoring)
    return FeatureSelectionResult(sfs, mask, idx, [feature_names[i] for i in idx] if feature_names else None,
                                  float(base.mean()), float(base.std()), float(sel.mean()), float(sel.std()))
