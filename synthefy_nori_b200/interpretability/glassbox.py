"""Glass-box distillation of a fitted Nori regressor.

Parity target: reference ``interpretability/glassbox`` (feature selection by the Nori
teacher, then an Explainable Boosting Machine fitted to the teacher's predictions and
scored on held-out rows; ``_core.py:190-300``, ``ebm.py:14-60``).  The reference's EBM
comes from the ``interpret`` package, which is not part of this environment; the
student here is the same model family written out: a generalised additive model with
one piecewise-constant shape function per selected feature (quantile bins), fitted by
cyclic gradient boosting on the teacher's predictions with a small learning rate
(Lou, Caruana & Gehrke, 2012), optionally with pairwise terms on a coarse 2-D grid.

Feature choice: permutation importance under the teacher (all permuted copies
predicted in one batch).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


def _edges(col: np.ndarray, bins: int) -> np.ndarray:
    col = col[np.isfinite(col)]
    e = np.unique(np.quantile(col, np.linspace(0, 1, bins + 1)[1:-1])) if len(col) else np.array([])
    return e


@dataclass
class GlassBoxModel:
    features: list
    edges: list
    shapes: list
    intercept: float
    pairs: list = field(default_factory=list)
    pair_shapes: list = field(default_factory=list)
    names: list | None = None

    def _codes(self, X: np.ndarray, k: int) -> np.ndarray:
        c = X[:, self.features[k]]
        return np.where(np.isfinite(c), np.searchsorted(self.edges[k], np.nan_to_num(c), side="right"),
                        len(self.edges[k]) + 1)

    def term_contributions(self, X) -> np.ndarray:
        X = np.asarray(X, np.float64)
        out = [self.shapes[k][self._codes(X, k)] for k in range(len(self.features))]
        for (a, b), sh in zip(self.pairs, self.pair_shapes):
            out.append(sh[np.minimum(self._codes(X, a), sh.shape[0] - 1), np.minimum(self._codes(X, b), sh.shape[1] - 1)])
        return np.stack(out, 1)

    def predict(self, X) -> np.ndarray:
        return self.intercept + self.term_contributions(X).sum(1)

    def importances(self, X) -> np.ndarray:
        return np.abs(self.term_contributions(X)).mean(0)


def permutation_importance(predict_fn, X: np.ndarray, n_repeats: int = 2, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    n, d = X.shape
    base = np.asarray(predict_fn(X), np.float64)
    blocks = []
    for j in range(d):
        for _ in range(n_repeats):
            Xp = X.copy()
            Xp[:, j] = X[rng.permutation(n), j]
            blocks.append(Xp)
    pred = np.asarray(predict_fn(np.concatenate(blocks).astype(np.float32)), np.float64).reshape(d, n_repeats, n)
    return ((pred - base[None, None]) ** 2).mean((1, 2))


def fit_gam(X: np.ndarray, target: np.ndarray, features: list, *, bins: int = 32, rounds: int = 300, lr: float = 0.1,
            interactions: int = 0, seed: int = 0) -> GlassBoxModel:
    X = np.asarray(X, np.float64)
    edges = [_edges(X[:, f], bins) for f in features]
    m = GlassBoxModel(list(features), edges, [np.zeros(len(e) + 2) for e in edges], float(target.mean()))
    codes = [m._codes(X, k) for k in range(len(features))]
    resid = target - m.intercept
    for _ in range(rounds):
        for k, c in enumerate(codes):
            nb = len(m.shapes[k])
            s = np.bincount(c, weights=resid, minlength=nb)
            cnt = np.bincount(c, minlength=nb)
            step = lr * np.divide(s, cnt, out=np.zeros(nb), where=cnt > 0)
            m.shapes[k] += step
            resid -= step[c]
    for k, c in enumerate(codes):  # centre each shape; the mean goes to the intercept
        mu = m.shapes[k][c].mean()
        m.shapes[k] -= mu
        m.intercept += mu
    if interactions:
        coarse = [np.minimum(c, 7) for c in codes]
        scores = []
        for a in range(len(features)):
            for b in range(a + 1, len(features)):
                key = coarse[a] * 8 + coarse[b]
                s = np.bincount(key, weights=resid, minlength=64)
                cnt = np.bincount(key, minlength=64)
                scores.append(((np.divide(s, cnt, out=np.zeros(64), where=cnt > 0) ** 2 * cnt).sum(), a, b))
        for _, a, b in sorted(scores, reverse=True)[:interactions]:
            key = coarse[a] * 8 + coarse[b]
            s = np.bincount(key, weights=resid, minlength=64)
            cnt = np.bincount(key, minlength=64)
            sh = np.divide(s, cnt, out=np.zeros(64), where=cnt > 0).reshape(8, 8)
            resid -= sh.reshape(-1)[key]
            m.pairs.append((a, b))
            m.pair_shapes.append(sh)
    return m


def distill_glassbox(regressor, X_train, X_test, y_test=None, *, n_features: int = 8, interactions: int = 0,
                     names=None, bins: int = 32, rounds: int = 300, seed: int = 0) -> dict:
    """Fit an additive student to a fitted ``NoriRegressor``'s predictions on ``X_train``;
    report the student's fidelity to the teacher and (with ``y_test``) both models' R^2."""
    Xtr, Xte = np.asarray(X_train, np.float32), np.asarray(X_test, np.float32)
    teacher_tr = np.asarray(regressor.predict(Xtr), np.float64)
    imp = permutation_importance(regressor.predict, Xtr[: min(len(Xtr), 512)], seed=seed)
    feats = sorted(np.argsort(-imp)[: min(n_features, Xtr.shape[1])].tolist())
    gam = fit_gam(Xtr, teacher_tr, feats, bins=bins, rounds=rounds, interactions=interactions, seed=seed)
    gam.names = [names[f] for f in feats] if names is not None else None
    teacher_te = np.asarray(regressor.predict(Xte), np.float64)
    student_te = gam.predict(Xte)

    def r2(t, p):
        ss = ((t - t.mean()) ** 2).sum()
        return float(1 - ((t - p) ** 2).sum() / ss) if ss > 0 else float("nan")

    rep = {"model": gam, "features": feats, "importance": imp, "fidelity_r2": r2(teacher_te, student_te)}
    if y_test is not None:
        y = np.asarray(y_test, np.float64)
        rep.update(teacher_r2=r2(y, teacher_te), student_r2=r2(y, student_te))
    return rep
