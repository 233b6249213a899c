"""Fitting and sampling for ``NoriRegressor`` with a 2-D target.

Parity target: reference ``api.py:672-803`` (fit: marginals, cross-fitted copula PITs,
autoregressive chains) and ``api.py:1014-1120`` (predict: ``"mean"`` from the
marginals' point predictions for the independent and copula strategies, otherwise the
mean of the joint draws; ``"samples"`` returns the draws ``[n, n_draws, n_targets]``).
"""

from __future__ import annotations

import numpy as np

from synthefy_nori_b200.multi_target import (MAX_AUTOREGRESSIVE_ROWS_PER_CALL, MULTI_TARGET_PREDICTION_STRATEGIES,
                                             GaussianCopula, MultiTargetPredictionPolicy, build_target_orders,
                                             cdf_from_quantile_bank, quantiles_from_levels)


class MultiTargetFit:
    def __init__(self, reg, Y: np.ndarray):
        strategy = reg.multi_target_prediction_strategy
        if strategy not in MULTI_TARGET_PREDICTION_STRATEGIES:
            raise ValueError(f"unknown multi_target_prediction_strategy {strategy!r}; expected one of "
                             f"{MULTI_TARGET_PREDICTION_STRATEGIES}")
        policy = MultiTargetPredictionPolicy.coerce(reg.multi_target_prediction_policy)
        if policy.autoregressive_orders is not None and strategy != "autoregressive":
            raise ValueError("autoregressive_orders requires multi_target_prediction_strategy='autoregressive'")
        if strategy == "copula" and policy.copula_cv > Y.shape[0]:
            raise ValueError(f"copula_cv cannot exceed the number of training rows ({Y.shape[0]})")
        if reg.discretize is not None or reg.categorical_levels is not None:
            raise ValueError("discretize and categorical_levels are not supported for multi-target regression")
        if reg.large_context_policy is not None:
            raise ValueError("large_context_policy is not supported for multi-target regression")
        self.reg, self.Y, self.strategy, self.policy = reg, Y, strategy, policy
        self.n_outputs = Y.shape[1]
        X = reg.X_train_
        if strategy in ("independent", "copula"):
            self.marginals = [reg._clone_for(X, Y[:, t]) for t in range(self.n_outputs)]
        if strategy == "copula":
            self._fit_copula()
        elif strategy == "autoregressive":
            self._fit_chains()

    def _fit_copula(self) -> None:
        from sklearn.model_selection import KFold

        pol, X, Y = self.policy, self.reg.X_train_, self.Y
        pits = np.empty_like(Y)
        for tr, va in KFold(pol.copula_cv, shuffle=True, random_state=pol.random_state).split(X):
            for t in range(self.n_outputs):
                d = self.reg._clone_for(X[tr], Y[tr, t])._distribution(X[va])
                pits[va, t] = cdf_from_quantile_bank(d["quantiles"], d["taus"], Y[va, t])
        pits = np.clip(pits, 1e-6, 1 - 1e-6)
        if pol.copula_pit_jitter > 0:
            rng = np.random.default_rng(pol.random_state)
            pits = np.clip(pits + rng.uniform(-pol.copula_pit_jitter, pol.copula_pit_jitter, pits.shape), 1e-6,
                           1 - 1e-6)
        self.copula = GaussianCopula().fit(pits)

    def _fit_chains(self) -> None:
        pol, X, Y = self.policy, self.reg.X_train_, self.Y
        if pol.autoregressive_orders is None:
            orders = build_target_orders(self.n_outputs, pol.autoregressive_n_orders, pol.random_state)
        else:
            orders = []
            for i, o in enumerate(pol.autoregressive_orders):
                if sorted(o) != list(range(self.n_outputs)):
                    raise ValueError(f"autoregressive_orders[{i}] must be a permutation of 0..{self.n_outputs - 1}")
                orders.append(np.asarray(o))
        self.orders = [tuple(int(t) for t in o) for o in orders]
        self.chains = [[self.reg._clone_for(X if k == 0 else np.concatenate([X, Y[:, list(o[:k])]], 1), Y[:, t])
                        for k, t in enumerate(o)] for o in self.orders]

    def predict(self, X: np.ndarray, *, output_type: str, quantiles, policy_override) -> np.ndarray:
        if output_type not in ("mean", "samples"):
            raise ValueError("multi-target regression supports output_type='mean' or 'samples'")
        if quantiles is not None:
            raise ValueError("quantiles= is not supported for multi-target regression; use output_type='samples'")
        pol = self.policy.merge_prediction_override(policy_override)
        if output_type == "mean" and self.strategy in ("independent", "copula"):
            return np.column_stack([m._point(X, self.reg.quantile_collapse) for m in self.marginals])
        draws = self.sample(X, pol)
        if not np.all(np.isfinite(draws)):
            raise RuntimeError("multi-target prediction produced non-finite samples")
        return draws if output_type == "samples" else draws.mean(1)

    def sample(self, X: np.ndarray, pol: MultiTargetPredictionPolicy) -> np.ndarray:
        rng = np.random.default_rng(pol.random_state)
        n, d, k = X.shape[0], self.n_outputs, pol.n_draws
        if self.strategy == "autoregressive":
            return self._sample_chains(X, pol, rng)
        U = (rng.random((n, k, d)) if self.strategy == "independent"
             else np.clip(self.copula.simulate(n * k, rng), 1e-6, 1 - 1e-6).reshape(n, k, d))
        out = np.empty_like(U)
        for t, m in enumerate(self.marginals):
            dist = m._distribution(X)
            out[:, :, t] = quantiles_from_levels(dist["quantiles"], dist["taus"], U[:, :, t])
        return out

    def _sample_chains(self, X, pol, rng) -> np.ndarray:
        n_orders = len(self.chains)
        base, extra = divmod(pol.n_draws, n_orders)
        parts = []
        for oi, (order, chain) in enumerate(zip(self.orders, self.chains)):
            cnt = base + (1 if oi < extra else 0)
            if cnt == 0:
                continue
            drawn = np.empty((X.shape[0], cnt, self.n_outputs))
            for pos, t in enumerate(order):
                if pos == 0:
                    dist = chain[0]._distribution(X)
                    drawn[:, :, t] = quantiles_from_levels(dist["quantiles"], dist["taus"],
                                                           rng.random((X.shape[0], cnt)))
                    continue
                prev = list(order[:pos])
                flat = drawn.reshape(X.shape[0] * cnt, self.n_outputs)
                for s in range(0, flat.shape[0], MAX_AUTOREGRESSIVE_ROWS_PER_CALL):
                    e = min(s + MAX_AUTOREGRESSIVE_ROWS_PER_CALL, flat.shape[0])
                    q = np.concatenate([X[np.arange(s, e) // cnt], flat[s:e][:, prev]], 1).astype(np.float32)
                    dist = chain[pos]._distribution(q)
                    flat[s:e, t] = quantiles_from_levels(dist["quantiles"], dist["taus"], rng.random((e - s, 1)))[:, 0]
            parts.append(drawn)
        return np.concatenate(parts, 1)
