"""Public local API: ``NoriRegressor`` (scikit-learn estimator) and one-shot helpers.

Parity target: reference ``src/synthefy_nori/api.py`` - ``NoriRegressor.__init__``
158-440 (parameters stored verbatim so ``clone`` round-trips), ``fit`` 464-619 (stores the
context, standardises y with the training mean / std), ``predict`` 862-968
(``output_type`` = mean | median | quantiles | full), ``infer`` / ``predict`` one-shot
helpers 1383-1478.  ``fit`` only stores rows; the context cache is built lazily on the
first ``predict`` and reused by later calls (the reference's context reuse cache).

Weights: ``model_path`` loads a reference-format checkpoint (``utils/loading.py``);
otherwise ``model`` names a preset and ``weights="random"`` builds a random-init model of
that architecture (there is no network access for the Hugging Face download here;
``synthefy_nori_b200.hf.download_checkpoint`` documents the hub path).
"""

from __future__ import annotations

import warnings
from typing import Literal

import numpy as np
import torch

try:
    from sklearn.base import BaseEstimator, RegressorMixin
except ImportError:  # pragma: no cover
    BaseEstimator, RegressorMixin = object, object

MODELS = ("nori-6m", "nori-1-5", "nori-30m", "nori-100m")


def _as_device(device) -> torch.device:
    if device is not None:
        return torch.device(device)
    if torch.cuda.is_available():
        return torch.device("cuda", torch.cuda.current_device())
    if getattr(torch.backends, "mps", None) is not None and torch.backends.mps.is_available():
        return torch.device("mps")
    return torch.device("cpu")


def _to_numpy_2d(X) -> np.ndarray:
    if hasattr(X, "to_numpy"):
        X = X.to_numpy(dtype=np.float32, na_value=np.nan)
    X = np.asarray(X, dtype=np.float32)
    if X.ndim == 1:
        X = X[:, None]
    if X.ndim != 2:
        raise ValueError("X must be 2-D")
    return X


class NoriRegressor(RegressorMixin, BaseEstimator):
    """In-context regression with a Nori model on the native B200 kernels.

    ``fit`` stores the context table; ``predict`` runs the query rows against a cached
    encoding of the context and returns point predictions, quantiles or the full
    999-quantile predictive distribution.
    """

    def __init__(
        self,
        model_path: str | None = None,
        *,
        model: str | None = None,
        device=None,
        weights: str | None = None,
        n_estimators: int = 1,
        cache_dtype: Literal["bf16", "int8"] | None = None,
        memory_policy=None,
        query_chunk_size: int | None = None,
        quantile_collapse: str = "mean",
        random_state: int = 0,
    ) -> None:
        self.model_path = model_path
        self.model = model
        self.device = device
        self.weights = weights
        self.n_estimators = n_estimators
        self.cache_dtype = cache_dtype
        self.memory_policy = memory_policy
        self.query_chunk_size = query_chunk_size
        self.quantile_collapse = quantile_collapse
        self.random_state = random_state

    # ------------------------------------------------------------------ model
    def _load_model(self):
        from synthefy_nori_b200.models.config import preset_config
        from synthefy_nori_b200.utils.loading import build_model, load_model

        if self.model_path is not None:
            return load_model(self.model_path)
        if self.model is None:
            raise ValueError("pass model_path=... or model=one of " + ", ".join(MODELS))
        if self.weights == "random":
            torch.manual_seed(self.random_state)
            m = build_model(preset_config(self.model))
            return m.eval()
        from synthefy_nori_b200.hf import download_checkpoint

        return load_model(download_checkpoint(model=self.model))

    def _get_predictor(self):
        from synthefy_nori_b200.inference.predictor import NoriPredictor

        if getattr(self, "predictor_", None) is None:
            model = self._load_model()
            dtype = self._resolve_memory(model)
            self.predictor_ = NoriPredictor(model, self.device_, n_estimators=self.n_estimators, cache_dtype=dtype,
                                            query_chunk_size=self.query_chunk_size, seed=self.random_state)
        return self.predictor_

    def _resolve_memory(self, model) -> str:
        """Pick the cache rung for this table (reference ``MemoryPolicy.resolve``)."""
        import math as _math

        from synthefy_nori_b200.inference.degradation import CacheQuantizedWarning, ContextSubsampledWarning
        from synthefy_nori_b200.inference.memory_policy import MemoryPolicy

        pol = MemoryPolicy.coerce(self.memory_policy)
        if self.cache_dtype is not None:
            pol = pol.model_copy(update={"cache_dtype": self.cache_dtype})
        if self.device_.type == "cuda":
            total = torch.cuda.get_device_properties(self.device_).total_memory / 1024 ** 3
        else:
            total = 64.0
        groups = _math.ceil(self.n_features_in_ / model.features_per_group) + 1
        pol = pol.resolve(n_context_rows=self.X_train_.shape[0], n_groups=groups, nlayers=model.nlayers,
                          embed_dim=model.embed_dim, head_dim=model.embed_dim // model.nhead, device_total_gb=total)
        self.memory_policy_ = pol
        if pol.rung == "subsample" and pol.dropped_context_rows > 0:
            warnings.warn(f"context subsampled: {pol.dropped_context_rows} rows dropped to fit the cache budget",
                          ContextSubsampledWarning, stacklevel=3)
            rng = np.random.default_rng(self.random_state)
            keep = np.sort(rng.choice(self.X_train_.shape[0], self.X_train_.shape[0] - pol.dropped_context_rows,
                                      replace=False))
            self.X_train_, self.y_train_ = self.X_train_[keep], self.y_train_[keep]
        dtype = "int8" if pol.rung in ("resident_int8", "context_sharded_int8") or pol.cache_dtype == "int8" else "bf16"
        if dtype == "int8" and pol.cache_dtype == "bf16":
            warnings.warn("context cache stored int8 to fit the memory budget", CacheQuantizedWarning, stacklevel=3)
        return dtype

    # ------------------------------------------------------------------ sklearn API
    def fit(self, X, y):
        X = _to_numpy_2d(X)
        y = np.asarray(y, dtype=np.float64).reshape(-1)
        if X.shape[0] != y.shape[0]:
            raise ValueError("X and y have different row counts")
        if X.shape[0] < 2:
            raise ValueError("need at least 2 context rows")
        if not np.all(np.isfinite(y)):
            raise ValueError("y must be finite")
        self.device_ = _as_device(self.device)
        self.X_train_ = X
        self.y_train_ = y
        self.y_mean_ = float(y.mean())
        std = float(y.std())
        self.y_std_ = std if std > 0 else 1.0
        self.n_features_in_ = X.shape[1]
        self.context_ = None
        self.predictor_ = None
        from synthefy_nori_b200.inference.memory_policy import MemoryPolicy

        MemoryPolicy.coerce(self.memory_policy)  # validate early (reference validates in fit)
        return self

    def _context(self):
        if getattr(self, "context_", None) is None:
            pred = self._get_predictor()
            yn = (self.y_train_ - self.y_mean_) / self.y_std_
            self.context_ = pred.fit_context(self.X_train_, yn.astype(np.float32))
        return self.context_

    def predict_distribution(self, X) -> dict:
        """Full predictive distribution: ascending quantiles ``[n, K]`` (y units), their
        levels ``taus [K]`` and the distribution mean ``[n]``."""
        X = _to_numpy_2d(X)
        pred = self._get_predictor()
        raw = pred.predict_raw(self._context(), X)
        mean, _, srt = pred.decode(raw, levels=[0.5], return_sorted=True)
        scale, shift = self.y_std_, self.y_mean_
        return {
            "quantiles": (srt * scale + shift).cpu().numpy(),
            "taus": pred.taus.cpu().numpy(),
            "mean": (mean * scale + shift).cpu().numpy(),
        }

    def predict(self, X, *, output_type: str = "mean", quantiles: list[float] | None = None):
        """``output_type``: ``"mean"`` (default), ``"median"``, ``"quantiles"`` (returns
        ``(len(quantiles), n)``) or ``"full"`` (dict, see ``predict_distribution``)."""
        if not hasattr(self, "X_train_"):
            raise RuntimeError("call fit() before predict()")
        X = _to_numpy_2d(X)
        if X.shape[1] != self.n_features_in_:
            raise ValueError(f"X has {X.shape[1]} features, the context has {self.n_features_in_}")
        if output_type == "full":
            return self.predict_distribution(X)
        pred = self._get_predictor()
        raw = pred.predict_raw(self._context(), X)
        scale, shift = self.y_std_, self.y_mean_
        if output_type == "mean":
            if self.quantile_collapse != "mean":
                warnings.warn("only quantile_collapse='mean' is implemented; using the mean", stacklevel=2)
            mean, _, _ = pred.decode(raw)
            return (mean * scale + shift).cpu().numpy()
        if output_type == "median":
            _, q, _ = pred.decode(raw, levels=[0.5])
            return (q[:, 0] * scale + shift).cpu().numpy()
        if output_type == "quantiles":
            if not quantiles:
                raise ValueError("output_type='quantiles' needs quantiles=[...] in (0, 1)")
            if any(not (0.0 < float(t) < 1.0) for t in quantiles):
                raise ValueError("quantile levels must lie in (0, 1)")
            _, q, _ = pred.decode(raw, levels=quantiles)
            return (q * scale + shift).T.cpu().numpy()
        if output_type == "mode":
            raise NotImplementedError("output_type='mode' is not implemented for the quantile head")
        raise ValueError(f"unknown output_type {output_type!r}")

    @property
    def memory_report_(self) -> dict:
        ctx = getattr(self, "context_", None)
        pol = getattr(self, "memory_policy_", None)
        rep = pol.describe() if pol is not None else {}
        rep.update({
            "cache_bytes": ctx.nbytes() if ctx is not None else 0,
            "context_rows": int(self.X_train_.shape[0]) if hasattr(self, "X_train_") else 0,
        })
        return rep


def infer(X_train, y_train, X_test, *, model: str = "nori-6m", output_type: str = "mean", quantiles=None, **kw):
    """One-shot ``fit`` + ``predict`` (reference ``api.py:1383``)."""
    return NoriRegressor(model=model, **kw).fit(X_train, y_train).predict(X_test, output_type=output_type,
                                                                         quantiles=quantiles)


def predict(X_train, y_train, X_test, **kw):
    """Alias of :func:`infer` (reference ``api.py:1443``)."""
    return infer(X_train, y_train, X_test, **kw)
