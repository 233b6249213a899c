"""Partial dependence and ICE curves (reference ``interpretability/pdp.py:14-60``).

Every (grid value, row) pair of a feature, or (grid cell, row) of a feature pair, is one
query row; all of them are predicted in one call against the fitted context.
"""

from __future__ import annotations

import numpy as np


def _grid(col: np.ndarray, n: int) -> np.ndarray:
    col = col[np.isfinite(col)]
    u = np.unique(col)
    if len(u) <= n:
        return u
    return np.unique(np.quantile(col, np.linspace(0.05, 0.95, n)))


def partial_dependence(estimator, X, features, *, kind: str = "average", grid_resolution: int = 20) -> dict:
    """``features``: an index or a ``(i, j)`` pair.  Returns ``{"grid_values", "average",
    "individual"}`` (``average`` shaped like the grid, ``individual`` ``[n_rows, ...]``)."""
    if kind not in ("average", "individual", "both"):
        raise ValueError("kind must be 'average', 'individual' or 'both'")
    X = np.asarray(X, np.float32)
    feats = (features,) if np.isscalar(features) else tuple(features)
    grids = [_grid(X[:, f], grid_resolution) for f in feats]
    mesh = np.array(list(np.ndindex(*[len(g) for g in grids])))
    rows = np.repeat(X[None], len(mesh), 0)
    for k, f in enumerate(feats):
        rows[:, :, f] = grids[k][mesh[:, k]][:, None]
    pred = np.asarray(estimator.predict(rows.reshape(-1, X.shape[1])), np.float64)
    pred = pred.reshape(len(mesh), X.shape[0]).T.reshape(X.shape[0], *[len(g) for g in grids])
    out = {"grid_values": grids, "features": feats}
    if kind in ("average", "both"):
        out["average"] = pred.mean(0)
    if kind in ("individual", "both"):
        out["individual"] = pred
    return out


def partial_dependence_plots(estimator, X, features, *, kind: str = "average", grid_resolution: int = 20, ax=None):
    """Plot 1-D curves (matplotlib, when installed); returns the computed curves."""
    res = [partial_dependence(estimator, X, f, kind="both", grid_resolution=grid_resolution) for f in features]
    try:
        import matplotlib.pyplot as plt
    except ImportError:
        return res
    axes = ax if ax is not None else plt.subplots(1, len(res), squeeze=False)[1][0]
    for a, r in zip(np.ravel(axes), res):
        if len(r["features"]) != 1:
            continue
        g = r["grid_values"][0]
        if kind in ("individual", "both"):
            a.plot(g, r["individual"].T, color="0.8", lw=0.5)
        if kind in ("average", "both"):
            a.plot(g, r["average"], lw=2)
        a.set_xlabel(f"feature {r['features'][0]}")
    return res
