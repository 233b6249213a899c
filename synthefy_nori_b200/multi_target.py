"""Joint prediction of several targets from per-target quantile banks.

Parity target: reference ``src/synthefy_nori/multi_target.py:18-200`` and
``api.py:672-803, 1014-1120``.  Three strategies:

- ``independent``: one marginal model per target; joint draws use independent uniforms.
- ``copula``: marginals as above plus a copula over the targets fitted on cross-fitted
  probability integral transforms (each training row's PIT comes from a model that did
  not see that row, ``copula_cv`` folds).  The reference fits an R-vine with
  ``pyvinecopulib``; that package is not part of this build's environment, so the copula
  here is Gaussian (normal scores of the PITs, their correlation matrix, sampling by
  Cholesky), the Gaussian member of the reference's pair-copula family set.
- ``autoregressive``: chains over target orders; position k conditions on the targets
  already drawn by appending them as features; draws are split over the orders.

Banks are inverted (``quantiles_from_levels``) and evaluated as CDFs
(``cdf_from_quantile_bank``) in batched tensor code.  ``MultiTargetPredictionPolicy``
keeps the reference's field names so configurations carry over.
"""

from __future__ import annotations

import math
from typing import Literal

import numpy as np
import torch
from pydantic import BaseModel, ConfigDict, Field, PositiveInt, model_validator

MULTI_TARGET_PREDICTION_STRATEGIES = ("independent", "copula", "autoregressive")
DEFAULT_MULTI_TARGET_PREDICTION_STRATEGY = "copula"
MAX_AUTOREGRESSIVE_ROWS_PER_CALL = 65536


class MultiTargetPredictionPolicy(BaseModel):
    model_config = ConfigDict(extra="forbid", frozen=True)

    n_draws: PositiveInt = Field(300, description="joint draws per query row")
    random_state: int | None = Field(0, ge=0, le=2 ** 32 - 1)
    copula_cv: int = Field(5, ge=2, description="cross-fitting folds for the copula PITs")
    copula_pit_jitter: float = Field(1e-4, ge=0.0)
    autoregressive_n_orders: PositiveInt = Field(3)
    autoregressive_orders: list[list[int]] | None = None

    @model_validator(mode="after")
    def _orders(self):
        if self.autoregressive_orders is None:
            return self
        if "autoregressive_n_orders" in self.model_fields_set:
            raise ValueError("autoregressive_orders cannot be combined with autoregressive_n_orders")
        if not self.autoregressive_orders or any(not o for o in self.autoregressive_orders):
            raise ValueError("autoregressive_orders must contain non-empty orders")
        keys = [tuple(o) for o in self.autoregressive_orders]
        if len(set(keys)) != len(keys):
            raise ValueError("autoregressive_orders must not repeat an order")
        return self

    @classmethod
    def coerce(cls, value) -> "MultiTargetPredictionPolicy":
        if value is None:
            return cls()
        if isinstance(value, cls):
            return value
        if isinstance(value, dict):
            return cls(**value)
        raise TypeError("multi_target_prediction_policy must be a MultiTargetPredictionPolicy, dict or None")

    def merge_prediction_override(self, override) -> "MultiTargetPredictionPolicy":
        if override is None:
            return self
        upd = self.coerce(override).model_dump(exclude_unset=True)
        merged = self.model_copy(update=upd)
        for f in ("copula_cv", "copula_pit_jitter", "autoregressive_n_orders", "autoregressive_orders"):
            if getattr(merged, f) != getattr(self, f):
                raise ValueError(f"multi_target_prediction_policy.{f} is fixed at fit time; refit instead")
        return merged


def cdf_from_quantile_bank(Q, taus, values) -> np.ndarray:
    """CDF of each row's piecewise-linear distribution at ``values`` (flat stretches are
    atoms: the CDF jumps across them; 0 below the bank, 1 at or above its top)."""
    Qt = torch.sort(torch.as_tensor(np.asarray(Q), dtype=torch.float64), dim=1).values
    t = torch.as_tensor(np.asarray(taus), dtype=torch.float64)
    y = torch.as_tensor(np.asarray(values), dtype=torch.float64).reshape(-1, 1)
    if Qt.dim() != 2 or Qt.shape[0] != y.shape[0] or Qt.shape[1] != t.numel() or t.numel() < 2:
        raise ValueError("quantile bank, tau levels and values have incompatible shapes")
    K = Qt.shape[1]
    lo_i = torch.searchsorted(Qt.contiguous(), y, right=False)  # first index with Q >= y
    hi_i = torch.searchsorted(Qt.contiguous(), y, right=True)  # first index with Q > y
    exact = hi_i > lo_i  # y equals one or more bank values: last level of the tie
    at = t[(hi_i - 1).clamp(0, K - 1)]
    j = lo_i.clamp(1, K - 1)
    q0, q1 = Qt.gather(1, j - 1), Qt.gather(1, j)
    w = ((y - q0) / (q1 - q0).clamp_min(1e-300)).clamp(0, 1)
    # below the upper tie group use its first level, above the lower one its last level
    hi_first = t[j]
    lo_last = t[(torch.searchsorted(Qt.contiguous(), q0, right=True) - 1).clamp(0, K - 1)]
    inner = (1 - w) * lo_last + w * hi_first
    out = torch.where(exact, at, inner)
    out = torch.where(y < Qt[:, :1], torch.zeros_like(out), out)
    out = torch.where(y >= Qt[:, -1:], torch.ones_like(out), out)
    return out.reshape(-1).numpy()


def quantiles_from_levels(Q, taus, U) -> np.ndarray:
    """Invert row-wise banks ``Q [n, K]`` at probability levels ``U [n, m]``."""
    Qt = torch.as_tensor(np.asarray(Q), dtype=torch.float64)
    t = torch.as_tensor(np.asarray(taus), dtype=torch.float64)
    u = torch.as_tensor(np.asarray(U), dtype=torch.float64)
    if Qt.dim() != 2 or u.dim() != 2 or Qt.shape[0] != u.shape[0] or Qt.shape[1] != t.numel() or t.numel() < 2:
        raise ValueError("quantile bank and probability levels have incompatible shapes")
    c = u.clamp(float(t[0]), float(t[-1]))
    hi = torch.searchsorted(t, c.contiguous(), right=True).clamp(1, t.numel() - 1)
    lo = hi - 1
    w = torch.where(t[hi] > t[lo], (c - t[lo]) / (t[hi] - t[lo]), torch.zeros_like(c))
    r = (1 - w) * Qt.gather(1, lo) + w * Qt.gather(1, hi)
    r = torch.where(c <= t[0], Qt[:, :1].expand_as(r), r)
    r = torch.where(c >= t[-1], Qt[:, -1:].expand_as(r), r)
    return r.numpy()


def build_target_orders(n_outputs: int, n_orders: int, random_state: int | None) -> list[np.ndarray]:
    """Identity first, then distinct random permutations (at most ``n_outputs!``)."""
    n_orders = min(n_orders, math.factorial(n_outputs))
    orders = [np.arange(n_outputs)]
    rng = np.random.default_rng(random_state)
    seen = {tuple(orders[0])}
    tries = 0
    while len(orders) < n_orders and tries < 50 * n_orders:
        tries += 1
        p = rng.permutation(n_outputs)
        if tuple(p) in seen:
            continue
        seen.add(tuple(p))
        orders.append(p)
    return orders


class GaussianCopula:
    """Gaussian copula fitted on PITs ``U [n, d]`` (normal scores -> correlation)."""

    def fit(self, U: np.ndarray) -> "GaussianCopula":
        from scipy.stats import norm

        Z = norm.ppf(np.clip(U, 1e-6, 1 - 1e-6))
        C = np.corrcoef(Z, rowvar=False) if Z.shape[1] > 1 else np.ones((1, 1))
        C = np.nan_to_num(C, nan=0.0)
        np.fill_diagonal(C, 1.0)
        w, V = np.linalg.eigh(C)  # nearest positive-definite correlation
        C = (V * np.clip(w, 1e-6, None)) @ V.T
        d = np.sqrt(np.diag(C))
        self.corr_ = C / np.outer(d, d)
        self.chol_ = np.linalg.cholesky(self.corr_)
        return self

    def simulate(self, n: int, rng: np.random.Generator) -> np.ndarray:
        from scipy.stats import norm

        z = rng.standard_normal((n, self.chol_.shape[0])) @ self.chol_.T
        return norm.cdf(z)


StrategyName = Literal["independent", "copula", "autoregressive"]
