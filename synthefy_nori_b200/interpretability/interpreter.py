"""``NoriInterpreter``: rank a table's features by a fitted Nori model, keep the fewest
that hold a set share of its skill, and fit an additive glass-box student on them.

Parity target: reference ``interpretability/glassbox/interpreter.py:48-487`` with
``_core.py:86-286`` and ``importance.py:17-98`` (fit on the full table with an internal
split, permutation or Shapley importance, a pruning sweep that stops at the first size
whose skill reaches ``retain`` of the full model's, a glass-box model on the kept
features plus an all-feature one, and the fitted attributes ``feature_importances_``,
``importance_ranking_``, ``selected_features_``, ``n_selected_``, ``sweep_``,
``nori_full_score_``, ``nori_selected_score_``, ``ebm_score_``, ``ebm_full_score_``,
``summary()``).  The reference's student is ``interpret``'s EBM; here it is this
package's own cyclic-boosted additive model (``glassbox.fit_gam``), kept under the same
attribute names (``ebm_``, ``ebm_full_``, ``ebm_model_``).

Tasks: regression (R^2), binary (ROC-AUC on the class-1 score), multiclass (mean
one-vs-rest ROC-AUC).  Classes are learned without inventing an order between them:
the teacher regresses one 0/1 indicator per class (one for binary) and the student is
one additive model per indicator.

Importance by permutation scores every shuffled copy of the evaluation rows in ONE
``predict`` call (one pass over the cached context for all features x repeats).
"""

from __future__ import annotations

import math

import numpy as np
from sklearn.base import BaseEstimator
from sklearn.metrics import r2_score, roc_auc_score
from sklearn.model_selection import train_test_split

from synthefy_nori_b200.interpretability.glassbox import fit_gam

# pruning sweep: fractions of the feature count tried in order (smallest first)
SWEEP = (0.02, 0.05, 0.08, 0.12, 0.18, 0.25, 0.35, 0.5, 0.7, 1.0)


def detect_task(y: np.ndarray, forced: str = "auto") -> str:
    if forced != "auto":
        if forced not in ("regression", "classification", "multiclass"):
            raise ValueError("task must be 'auto', 'regression', 'classification' or 'multiclass'")
        return forced
    if y.dtype.kind in "OUSb":
        return "classification" if len(np.unique(y)) == 2 else "multiclass"
    vals = np.unique(y[np.isfinite(y)])
    if len(vals) == 2:
        return "classification"
    if len(vals) <= 20 and np.all(vals == np.round(vals)):
        return "multiclass"
    return "regression"


def _auc(y: np.ndarray, s: np.ndarray) -> float:
    if s.ndim == 1:
        return float(roc_auc_score(y, s))
    per = [roc_auc_score(y == k, s[:, k]) for k in range(s.shape[1]) if 0 < (y == k).sum() < len(y)]
    if not per:
        raise ValueError("no class has both positive and negative rows in the evaluation split")
    return float(np.mean(per))


def metric_for(task: str):
    return (r2_score, "r2") if task == "regression" else (_auc, "roc_auc")


def retain_target(task: str, full: float, retain: float) -> float:
    """Skill a reduced feature set must reach: ``retain`` of the full model's skill above
    chance (R^2 0, AUC 0.5)."""
    floor = 0.0 if task == "regression" else 0.5
    return floor + retain * (full - floor) if full > floor else full


class _Teacher:
    """A Nori regressor per target column: the value (regression) or each class's 0/1
    indicator (classification: one column for binary, K for multiclass)."""

    def __init__(self, template, task: str, n_classes: int):
        from sklearn.base import clone

        self.task = task
        cols = 1 if task != "multiclass" else n_classes
        self.models = [clone(template) for _ in range(cols)]

    def fit(self, X, y):
        if self.task == "regression":
            self.models[0].fit(X, y.astype(np.float32))
        elif self.task == "classification":
            self.models[0].fit(X, (y == 1).astype(np.float32))
        else:
            for k, m in enumerate(self.models):
                m.fit(X, (y == k).astype(np.float32))
        return self

    def predict(self, X):
        out = [np.asarray(m.predict(X), np.float64) for m in self.models]
        return out[0] if len(out) == 1 else np.stack(out, 1)


class _Student:
    """Additive model(s) on the kept columns; one per teacher output column."""

    def __init__(self, X, y, task: str, n_classes: int, names, *, bins, rounds, interactions, seed):
        cols = list(range(X.shape[1]))
        if task == "regression":
            targets = [y.astype(np.float64)]
        elif task == "classification":
            targets = [(y == 1).astype(np.float64)]
        else:
            targets = [(y == k).astype(np.float64) for k in range(n_classes)]
        self.gams = [fit_gam(X, t, cols, bins=bins, rounds=rounds, interactions=interactions, seed=seed)
                     for t in targets]
        for g in self.gams:
            g.names = list(names)

    def predict(self, X):
        out = [g.predict(X) for g in self.gams]
        return out[0] if len(out) == 1 else np.stack(out, 1)

    def structure(self) -> dict:
        g = self.gams[0]
        return {"intercept": [float(m.intercept) for m in self.gams], "features": list(g.names),
                "term_edges": [e.tolist() for e in g.edges],
                "shapes": [[s.tolist() for s in m.shapes] for m in self.gams],
                "pairs": [list(p) for p in g.pairs]}


def permutation_importance_skill(model, X, y, metric, *, n_repeats: int = 3, seed: int = 0):
    """Skill drop per column when it is shuffled; all shuffled copies predicted together."""
    rng = np.random.default_rng(seed)
    n, d = X.shape
    base = metric(y, model.predict(X))
    copies = []
    for j in range(d):
        for _ in range(n_repeats):
            Xp = X.copy()
            Xp[:, j] = X[rng.permutation(n), j]
            copies.append(Xp)
    pred = model.predict(np.concatenate(copies))
    pred = pred.reshape((d, n_repeats, n) + pred.shape[1:])
    drop = np.array([[base - metric(y, pred[j, r]) for r in range(n_repeats)] for j in range(d)])
    return drop.mean(1), float(base)


def shap_importance(model, X, background, *, budget: int = 256, seed: int = 0, imputer: str = "baseline"):
    """Mean |Shapley value| per column over the rows of ``X`` (first teacher column)."""
    from synthefy_nori_b200.interpretability.shapley import ImputationExplainer

    def f(rows):
        p = model.predict(rows)
        return p if p.ndim == 1 else p[:, -1]

    ex = ImputationExplainer(f, background, index="SV", max_order=1, random_state=seed, imputer=imputer)
    d = X.shape[1]
    acc = np.zeros(d)
    for row in X:
        acc += np.abs(ex.explain(row, budget=budget).values_array(d))
    return acc / max(len(X), 1)


class NoriInterpreter(BaseEstimator):
    """See the module docstring.  ``model`` is a preset name or a ``NoriRegressor`` to
    clone; ``regressor_kwargs`` go to ``NoriRegressor`` when a name is given."""

    def __init__(self, model="nori-6m", *, task: str = "auto", method: str = "permutation", test_size: float = 0.3,
                 use_test: bool = True, reduce_threshold: int = 16, retain: float = 0.95, n_repeats: int = 3,
                 perm_eval: int = 2000, shap_rows: int = 32, shap_budget: int = 256, context_cap: int = 10_000,
                 interactions: int = 0, bins: int = 32, rounds: int = 300, random_state: int = 0,
                 regressor_kwargs: dict | None = None, verbose: bool = False):
        self.model = model
        self.task = task
        self.method = method
        self.test_size = test_size
        self.use_test = use_test
        self.reduce_threshold = reduce_threshold
        self.retain = retain
        self.n_repeats = n_repeats
        self.perm_eval = perm_eval
        self.shap_rows = shap_rows
        self.shap_budget = shap_budget
        self.context_cap = context_cap
        self.interactions = interactions
        self.bins = bins
        self.rounds = rounds
        self.random_state = random_state
        self.regressor_kwargs = regressor_kwargs
        self.verbose = verbose

    # ------------------------------------------------------------------ helpers
    def _template(self):
        from synthefy_nori_b200.api import NoriRegressor

        if isinstance(self.model, str):
            return NoriRegressor(model=self.model, **(self.regressor_kwargs or {}))
        return self.model

    def _say(self, msg: str) -> None:
        if self.verbose:
            print(msg, flush=True)

    def _teacher(self, X, y):
        return _Teacher(self._template(), self.task_, self.n_classes_).fit(X, y)

    # ------------------------------------------------------------------ fit
    def fit(self, X, y, feature_names=None):
        if feature_names is None and hasattr(X, "columns"):
            feature_names = [str(c) for c in X.columns]
        X = np.asarray(X, np.float32)
        y = np.asarray(y)
        d = X.shape[1]
        names = list(feature_names) if feature_names is not None else [f"f{j}" for j in range(d)]
        if len(names) != d:
            raise ValueError(f"{len(names)} feature names for {d} columns")
        if self.method not in ("permutation", "shap"):
            raise ValueError("method must be 'permutation' or 'shap'")
        task = detect_task(y, self.task)
        self.task_ = task
        if task == "regression":
            self.classes_, yc, self.n_classes_ = None, y.astype(np.float64), 1
        else:
            self.classes_, yc = np.unique(y, return_inverse=True)
            self.n_classes_ = len(self.classes_)
            if task == "classification" and self.n_classes_ != 2:
                raise ValueError(f"binary classification needs 2 classes, got {self.n_classes_}")
        metric, metric_name = metric_for(task)
        strat = yc if task != "regression" else None
        Xtr, Xte, ytr, yte = train_test_split(X, yc, test_size=self.test_size, random_state=self.random_state,
                                              stratify=strat)
        # column means of the training split stand in for missing values of the student
        self._impute_mu_ = np.nan_to_num(np.nanmean(np.where(np.isfinite(Xtr), Xtr, np.nan), 0))
        rng = np.random.default_rng(self.random_state)
        if len(Xtr) > self.context_cap:  # the teacher's context is capped; the student sees every row
            keep = np.sort(rng.choice(len(Xtr), self.context_cap, replace=False))
            ctx_X, ctx_y = Xtr[keep], ytr[keep]
        else:
            ctx_X, ctx_y = Xtr, ytr
        if self.use_test:  # importance and sweep read the test split (post-hoc reading)
            fit_X, fit_y, ev_X, ev_y = ctx_X, ctx_y, Xte, yte
        else:  # nothing that chooses features sees the test split
            fit_X, ev_X, fit_y, ev_y = train_test_split(ctx_X, ctx_y, test_size=self.test_size,
                                                        random_state=self.random_state, stratify=(
                                                            ctx_y if task != "regression" else None))
        teacher = self._teacher(fit_X, fit_y)
        if len(ev_X) > self.perm_eval:
            take = rng.choice(len(ev_X), self.perm_eval, replace=False)
            imp_X, imp_y = ev_X[take], ev_y[take]
        else:
            imp_X, imp_y = ev_X, ev_y
        if self.method == "permutation":
            importance, base = permutation_importance_skill(teacher, imp_X, imp_y, metric, n_repeats=self.n_repeats,
                                                            seed=self.random_state)
        else:
            rows = imp_X[rng.choice(len(imp_X), min(self.shap_rows, len(imp_X)), replace=False)]
            importance = shap_importance(teacher, rows, fit_X, budget=self.shap_budget, seed=self.random_state)
            base = metric(imp_y, teacher.predict(imp_X))
        order = [int(j) for j in np.argsort(-importance, kind="stable")]
        full = float(metric(ev_y, teacher.predict(ev_X)))
        target = retain_target(task, full, self.retain)
        reduced = d > self.reduce_threshold
        sweep, n_sel, sel_score, sel_model = [], d, full, teacher
        if reduced:
            for k in sorted({max(1, math.ceil(f * d)) for f in SWEEP}):
                cols = order[:k]
                m = teacher if k == d else self._teacher(fit_X[:, cols], fit_y)
                s = float(metric(ev_y, m.predict(ev_X[:, cols])))
                sweep.append({"k": k, metric_name: round(s, 4)})
                self._say(f"  top {k:>4}/{d:<4} {metric_name}={s:+.4f} (target {target:+.4f})")
                if s >= target:
                    n_sel, sel_score, sel_model = k, s, m
                    break
        cols = order[:n_sel] if reduced else list(range(d))
        # test-split scores of the teacher (refit on the capped training rows when the
        # selection fit held part of them out)
        if self.use_test:
            nori_full, nori_sel, final_full = full, sel_score, teacher
        else:
            final_full = self._teacher(ctx_X, ctx_y)
            nori_full = float(metric(yte, final_full.predict(Xte)))
            nori_sel = nori_full if not reduced else float(
                metric(yte, self._teacher(ctx_X[:, cols], ctx_y).predict(Xte[:, cols])))
        # glass-box students on every training row
        Xs = np.where(np.isfinite(Xtr), Xtr, self._impute_mu_[None, :]).astype(np.float64)
        Xs_te = np.where(np.isfinite(Xte), Xte, self._impute_mu_[None, :]).astype(np.float64)
        kw = dict(bins=self.bins, rounds=self.rounds, interactions=self.interactions, seed=self.random_state)
        student = _Student(Xs[:, cols], ytr, task, self.n_classes_, [names[c] for c in cols], **kw)
        st_score = float(metric(yte, student.predict(Xs_te[:, cols])))
        if reduced:
            student_all = _Student(Xs, ytr, task, self.n_classes_, names, **kw)
            st_all_score = float(metric(yte, student_all.predict(Xs_te)))
        else:
            student_all, st_all_score = student, st_score

        self.metric_ = metric_name
        self.feature_names_ = names
        self.feature_importances_ = np.asarray(importance, np.float64)
        self.importance_ranking_ = [{"feature": names[j], "index": j, "importance": float(importance[j])}
                                    for j in order]
        self.selected_indices_ = [int(c) for c in cols]
        self.selected_features_ = [names[c] for c in cols]
        self.n_selected_ = len(cols)
        self.reduced_ = reduced
        self.base_score_ = float(base)
        self.sweep_ = sweep
        self.selection_score_ = float(sel_score)
        self.selection_full_score_ = full
        self.retain_target_ = float(target)
        self.nori_full_score_ = nori_full
        self.nori_selected_score_ = nori_sel
        self.ebm_score_ = st_score
        self.ebm_full_score_ = st_all_score
        self.nori_ = final_full
        self.nori_selected_ = sel_model
        self.ebm_ = student
        self.ebm_full_ = student_all
        self.ebm_model_ = student.structure()
        return self

    # ------------------------------------------------------------------ use
    def _prep(self, X):
        X = np.asarray(X, np.float64)
        X = np.where(np.isfinite(X), X, self._impute_mu_[None, :])
        return X[:, self.selected_indices_]

    def decision_function(self, X) -> np.ndarray:
        return self.ebm_.predict(self._prep(X))

    def predict(self, X) -> np.ndarray:
        """The glass-box student's prediction on the kept columns (class labels for
        classification)."""
        s = self.decision_function(X)
        if self.task_ == "regression":
            return s
        if self.task_ == "classification":
            return self.classes_[(s >= 0.5).astype(int)]
        return self.classes_[s.argmax(1)]

    def predict_proba(self, X) -> np.ndarray:
        if self.task_ == "regression":
            raise AttributeError("predict_proba is defined for classification tasks only")
        s = np.clip(self.decision_function(X), 0.0, None)
        if self.task_ == "classification":
            p1 = np.clip(s, 0.0, 1.0)
            return np.stack([1 - p1, p1], 1)
        tot = s.sum(1, keepdims=True)
        return np.where(tot > 0, s / np.where(tot > 0, tot, 1.0), 1.0 / s.shape[1])

    def plot_model(self, *, out_path: str | None = None, target_name: str | None = None):
        """One panel per kept feature with the student's shape function."""
        try:
            import matplotlib

            matplotlib.use("Agg")
            import matplotlib.pyplot as plt
        except ImportError as exc:  # optional extra
            raise ImportError("plot_model needs matplotlib") from exc
        g = self.ebm_.gams[0]
        k = len(g.features)
        fig, axes = plt.subplots(1, k, figsize=(3 * k, 2.6), squeeze=False)
        for i, ax in enumerate(axes[0]):
            e = g.edges[i]
            xs = np.concatenate([[e[0] - 1 if len(e) else -1], e]) if len(e) else np.array([0.0])
            ax.step(xs, g.shapes[i][: len(xs)], where="post")
            ax.set_title(g.names[i])
        fig.suptitle(target_name or "glass-box shape functions")
        if out_path:
            fig.savefig(out_path)
        return fig

    def summary(self) -> dict:
        return {"task": self.task_, "metric": self.metric_, "n_features": len(self.feature_names_),
                "n_selected": self.n_selected_, "reduced": self.reduced_, "retain_target": self.retain_target_,
                "nori_full": self.nori_full_score_, "nori_selected": self.nori_selected_score_,
                "ebm_selected": self.ebm_score_, "ebm_full": self.ebm_full_score_,
                "top_features": [r["feature"] for r in self.importance_ranking_[:10]], "sweep": self.sweep_}
