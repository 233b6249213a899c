"""Shapley attributions by baseline imputation.

Parity target: reference ``interpretability/shapiq.py:105-148`` (an imputation explainer
over a fitted ``NoriRegressor``: features outside a coalition are replaced by the
background's mean, or its most common value for categorical features; ``index="SV"``
Shapley values or order-2 interactions).  The reference delegates to ``shapiq``; this
build computes the indices itself:

- ``SV``: exact enumeration of all ``2^d`` coalitions when that fits the ``budget``,
  otherwise Kernel SHAP (Lundberg & Lee, 2017): coalitions sampled by the Shapley kernel
  ``(d-1) / (C(d,|S|) |S| (d-|S|))`` over sizes, solved by weighted least squares with
  the efficiency constraint (values sum to ``f(x) - f(baseline)``).
- ``SII`` (order 2, exact, ``d <= 14``): the pairwise Shapley interaction index
  ``sum_S |S|!(d-|S|-2)!/(d-1)! [f(S+ij) - f(S+i) - f(S+j) + f(S)]``.

Imputers (what a feature outside the coalition takes):

- ``baseline``: the background mean (most common value for categorical features); one
  model row per coalition;
- ``marginal``: ``n_samples`` background rows drawn once per explainer; the coalition's
  value is the mean prediction over them (interventional Shapley values);
- ``conditional``: per coalition, the ``n_samples`` background rows nearest to ``x`` in
  the coalition's own features (standardised Euclidean distance) supply the absent
  features, a nearest-neighbour estimate of the conditional distribution (the reference's
  ``shapiq`` conditional imputer fits a generative model for the same purpose).

All coalition rows of one explanation (coalitions x samples) go to the model as one query
batch.
"""

from __future__ import annotations

import itertools
import math

import numpy as np


class InteractionValues(dict):
    """``{(i,): value, (i, j): value, (): baseline}`` with helpers."""

    def values_array(self, d: int) -> np.ndarray:
        return np.array([self.get((i,), 0.0) for i in range(d)])


class ImputationExplainer:
    def __init__(self, predict_fn, background: np.ndarray, *, categorical_features=(), index: str = "SV",
                 max_order: int = 1, random_state: int | None = 0, imputer: str = "baseline", n_samples: int = 16):
        if index not in ("SV", "SII", "k-SII"):
            raise ValueError("index must be 'SV', 'SII' or 'k-SII'")
        if imputer not in ("baseline", "marginal", "conditional"):
            raise ValueError("imputer must be 'baseline', 'marginal' or 'conditional'")
        self.predict_fn = predict_fn
        self.imputer = imputer
        bg = np.asarray(background, np.float64)
        base = np.nanmean(bg, 0)
        for c in categorical_features:
            vals, cnt = np.unique(bg[:, c][np.isfinite(bg[:, c])], return_counts=True)
            if len(vals):
                base[c] = vals[cnt.argmax()]
        self.baseline = np.nan_to_num(base)
        self.index = "SV" if (index == "k-SII" and max_order == 1) else index
        self.max_order = 2 if self.index in ("SII", "k-SII") else 1
        self.rng = np.random.default_rng(random_state)
        fill = np.where(np.isfinite(bg), bg, self.baseline[None, :])
        if imputer == "marginal":
            take = self.rng.choice(len(fill), size=min(n_samples, len(fill)), replace=False)
            self.samples = fill[take]
        else:
            self.samples = fill
        self.n_samples = min(int(n_samples), len(fill))
        sd = fill.std(0)
        self._inv_sd = np.where(sd > 0, 1.0 / np.where(sd > 0, sd, 1.0), 0.0)

    def _eval(self, x: np.ndarray, masks: np.ndarray) -> np.ndarray:
        if self.imputer == "baseline":
            rows = np.where(masks, x[None, :], self.baseline[None, :]).astype(np.float32)
            return np.asarray(self.predict_fn(rows), np.float64).reshape(-1)
        S = self.n_samples
        if self.imputer == "marginal":
            donors = np.broadcast_to(self.samples[None], (len(masks), S, x.size))
        else:  # nearest background rows in the coalition's standardised features
            diff = ((self.samples - x[None, :]) * self._inv_sd[None, :]) ** 2  # [n_bg, d]
            dist = masks.astype(np.float64) @ diff.T  # [n_masks, n_bg]
            near = np.argpartition(dist, S - 1, axis=1)[:, :S] if S < dist.shape[1] else \
                np.broadcast_to(np.arange(dist.shape[1]), dist.shape)
            donors = self.samples[near]  # [n_masks, S, d]
        rows = np.where(masks[:, None, :], x[None, None, :], donors).reshape(-1, x.size).astype(np.float32)
        return np.asarray(self.predict_fn(rows), np.float64).reshape(len(masks), S).mean(1)

    def explain(self, x, budget: int = 2048) -> InteractionValues:
        x = np.asarray(x, np.float64).reshape(-1)
        d = x.size
        if self.max_order == 2:
            if d > 14:
                raise ValueError("exact order-2 interactions are limited to 14 features")
            return self._sii(x, d)
        if 2 ** d <= budget:
            return self._exact_sv(x, d)
        return self._kernel_sv(x, d, budget)

    def _exact_sv(self, x, d) -> InteractionValues:
        masks = np.array(list(itertools.product([False, True], repeat=d)))
        f = dict(zip(map(lambda m: m.tobytes(), masks), self._eval(x, masks)))
        phi = np.zeros(d)
        for m in masks:
            s = int(m.sum())
            for i in np.flatnonzero(~m):
                w = math.factorial(s) * math.factorial(d - s - 1) / math.factorial(d)
                m2 = m.copy()
                m2[i] = True
                phi[i] += w * (f[m2.tobytes()] - f[m.tobytes()])
        out = InteractionValues({(i,): phi[i] for i in range(d)})
        out[()] = f[np.zeros(d, bool).tobytes()]
        return out

    def _kernel_sv(self, x, d, budget) -> InteractionValues:
        sizes = np.arange(1, d)
        kw = (d - 1) / (np.array([math.comb(d, int(s)) for s in sizes]) * sizes * (d - sizes))
        p = kw * np.array([math.comb(d, int(s)) for s in sizes])
        p /= p.sum()
        n = max(budget - 2, 2 * d)
        masks = np.zeros((n, d), bool)
        for r, s in enumerate(self.rng.choice(sizes, size=n, p=p)):
            masks[r, self.rng.choice(d, size=s, replace=False)] = True
        ends = np.array([np.zeros(d, bool), np.ones(d, bool)])
        f = self._eval(x, np.concatenate([ends, masks]))
        f0, f1, fm = f[0], f[1], f[2:]
        # constrained weighted least squares (samples drawn from the kernel -> unit weights)
        Z = masks.astype(np.float64)
        yv = fm - f0
        total = f1 - f0
        # eliminate the last coordinate with the efficiency constraint
        A = Z[:, :-1] - Z[:, -1:]
        b = yv - Z[:, -1] * total
        phi_head = np.linalg.lstsq(A, b, rcond=None)[0]
        phi = np.append(phi_head, total - phi_head.sum())
        out = InteractionValues({(i,): phi[i] for i in range(d)})
        out[()] = f0
        return out

    def _sii(self, x, d) -> InteractionValues:
        masks = np.array(list(itertools.product([False, True], repeat=d)))
        code = masks @ (1 << np.arange(d))
        f = np.empty(1 << d)
        f[code] = self._eval(x, masks)
        out = self._exact_sv(x, d)
        for i, j in itertools.combinations(range(d), 2):
            acc = 0.0
            for c in range(1 << d):
                if c >> i & 1 or c >> j & 1:
                    continue
                s = bin(c).count("1")
                w = math.factorial(s) * math.factorial(d - s - 2) / math.factorial(d - 1)
                acc += w * (f[c | 1 << i | 1 << j] - f[c | 1 << i] - f[c | 1 << j] + f[c])
            out[(i, j)] = acc
        return out


def get_nori_imputation_explainer(model, data, *, index: str = "k-SII", max_order: int = 2, imputer: str = "baseline",
                                  random_state: int | None = 0, n_samples: int = 16) -> ImputationExplainer:
    """Explainer over a fitted ``NoriRegressor`` with ``data`` as the background;
    ``imputer`` is ``"baseline"`` (one row per coalition, the fastest), ``"marginal"`` or
    ``"conditional"`` (``n_samples`` rows per coalition)."""
    cats = list(getattr(model, "categorical_features_", []) or [])
    return ImputationExplainer(lambda rows: model.predict(rows), data, categorical_features=cats, index=index,
                               max_order=max_order, random_state=random_state, imputer=imputer, n_samples=n_samples)
