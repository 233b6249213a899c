"""Public local API: ``NoriRegressor`` (scikit-learn estimator) and one-shot helpers.

Parity target: reference ``src/synthefy_nori/api.py``: ``NoriRegressor.__init__``
158-440 (parameters stored verbatim so ``clone`` round-trips), ``fit`` 464-619 (device
resolution CUDA -> MPS -> CPU, DataFrame preprocessing, identifier encoding, y
standardised with the training mean / std, multi-target routing), ``predict`` 862-968
(``output_type`` = mean | median | mode | quantiles | full, ``discretize=`` /
``categorical_levels=``), ``get_embeddings`` 1220-1254, the Yeo-Johnson second pass for
heavily skewed targets (``inference/predictor.py:1874-2003``), large-context policies,
and the ``infer`` / ``predict`` one-shot helpers 1383-1478.  ``fit`` only stores rows;
the context cache is built on the first ``predict`` and reused by later calls.

Weights: ``model_path`` loads a reference-format checkpoint (``utils/loading.py``);
otherwise ``model`` names a preset and ``weights="random"`` builds a random-init model of
that architecture (``synthefy_nori_b200.hf.download_checkpoint`` fetches released
weights where the hub is reachable).
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
YJ_SKEW_THRESHOLD = 10.0


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
    encoding of the context and returns point predictions, quantiles, the full
    999-quantile predictive distribution, or labels on a discrete target's lattice.
    A 2-D ``y`` fits several targets jointly (``multi_target_prediction_strategy``).
    """

    def __init__(
        self,
        model_path: str | None = None,
        *,
        model: str | None = None,
        device=None,
        weights: str | None = None,
        n_estimators: int | None = None,
        inference_config=None,
        cache_dtype: Literal["bf16", "int8"] | None = None,
        memory_policy=None,
        query_chunk_size: int | None = None,
        quantile_collapse: str = "mean",
        bar_point_estimator: str = "mean",
        discretize: str | None = None,
        categorical_levels=None,
        categorical_columns="auto",
        text_columns=None,
        categorical_encoding: str = "ordinal",
        max_categorical_cardinality: int = 100,
        encode_id_cols: list[str] | None = None,
        augmentations: tuple[str, ...] = ("yj",),
        yj_skew_threshold: float = YJ_SKEW_THRESHOLD,
        multi_target_prediction_strategy: str = "copula",
        multi_target_prediction_policy=None,
        large_context_policy=None,
        large_context_threshold: int | None = None,
        large_context_window: int | None = None,
        random_state: int = 0,
    ) -> None:
        self.model_path = model_path
        self.model = model
        self.device = device
        self.weights = weights
        self.n_estimators = n_estimators
        self.inference_config = inference_config
        self.cache_dtype = cache_dtype
        self.memory_policy = memory_policy
        self.query_chunk_size = query_chunk_size
        self.quantile_collapse = quantile_collapse
        self.bar_point_estimator = bar_point_estimator
        self.discretize = discretize
        self.categorical_levels = categorical_levels
        self.categorical_columns = categorical_columns
        self.text_columns = text_columns
        self.categorical_encoding = categorical_encoding
        self.max_categorical_cardinality = max_categorical_cardinality
        self.encode_id_cols = encode_id_cols
        self.augmentations = augmentations
        self.yj_skew_threshold = yj_skew_threshold
        self.multi_target_prediction_strategy = multi_target_prediction_strategy
        self.multi_target_prediction_policy = multi_target_prediction_policy
        self.large_context_policy = large_context_policy
        self.large_context_threshold = large_context_threshold
        self.large_context_window = large_context_window
        self.random_state = random_state

    # ------------------------------------------------------------------ model
    def _load_model(self):
        from synthefy_nori_b200.models.config import preset_config
        from synthefy_nori_b200.utils.loading import build_model, load_model

        if getattr(self, "_model_obj", None) is not None:
            return self._model_obj
        if self.model_path is not None:
            m = load_model(self.model_path)
        elif self.model is None:
            raise ValueError("pass model_path=... or model=one of " + ", ".join(MODELS))
        elif self.weights == "random":
            torch.manual_seed(self.random_state)
            m = build_model(preset_config(self.model)).eval()
        else:
            from synthefy_nori_b200.hf import download_checkpoint

            m = load_model(download_checkpoint(model=self.model))
        self._model_obj = m
        return m

    def _get_predictor(self):
        from synthefy_nori_b200.inference.predictor import NoriPredictor

        if getattr(self, "predictor_", None) is None:
            model = self._load_model()
            if getattr(self, "memory_policy_", None) is None or self.memory_policy_.rung is None:
                self._resolve_memory(model)
            pol = self.memory_policy_
            dtype, placement, block_rows = pol.placement()
            self.predictor_ = NoriPredictor(model, self.device_, inference_config=self.inference_config,
                                            n_estimators=self.n_estimators, cache_dtype=dtype,
                                            query_chunk_size=self.query_chunk_size, seed=self.random_state,
                                            reuse_context_cache=pol.reuse_context_cache, placement=placement,
                                            stream_block_rows=block_rows)
        return self.predictor_

    def _escalate_memory(self, exc) -> bool:
        """After an out-of-memory error: move the policy to its next rung (warning) and
        drop the predictor so the next attempt rebuilds the cache there."""
        from synthefy_nori_b200.inference.degradation import MemoryEscalatedWarning

        pol = getattr(self, "memory_policy_", None)
        nxt = pol.next_rung() if pol is not None else None
        if nxt is None:
            return False
        warnings.warn(f"out of GPU memory on the {pol.rung} cache rung; retrying on {nxt}", MemoryEscalatedWarning,
                      stacklevel=4)
        self.memory_policy_ = pol.escalated(nxt)
        self.predictor_ = None
        self.context_ = self.context_yj_ = None
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
        return True

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
        dtype = pol.placement()[0]
        if dtype == "int8" and pol.cache_dtype == "bf16":
            warnings.warn("context cache stored int8 to fit the memory budget", CacheQuantizedWarning, stacklevel=3)
        return dtype

    # ------------------------------------------------------------------ features
    def _fit_features(self, X) -> np.ndarray:
        self.categorical_features_ = []
        self.id_encoder_ = self.frame_preprocessor_ = None
        if hasattr(X, "columns") and hasattr(X, "dtypes"):
            from synthefy_nori_b200.featurize import DataFramePreprocessor

            if self.encode_id_cols:
                from synthefy_nori_b200.entity_ids import EntityIDPreprocessor

                self.id_encoder_ = EntityIDPreprocessor(list(self.encode_id_cols))
                X = self.id_encoder_.fit_transform(X)
            self.frame_preprocessor_ = DataFramePreprocessor(
                categorical_columns=self.categorical_columns, text_columns=self.text_columns,
                max_categorical_cardinality=self.max_categorical_cardinality,
                categorical_encoding=self.categorical_encoding)
            out = self.frame_preprocessor_.fit_transform(X)
            if self.categorical_encoding == "ordinal":
                cats = set(self.frame_preprocessor_.categorical_columns_)
                self.categorical_features_ = [i for i, c in enumerate(out.columns) if c in cats]
            self.feature_names_in_ = np.asarray(X.columns, dtype=object)
            return out.to_numpy(np.float32)
        if self.encode_id_cols:
            raise ValueError("encode_id_cols requires a DataFrame")
        return _to_numpy_2d(X)

    def _query_features(self, X) -> np.ndarray:
        if getattr(self, "frame_preprocessor_", None) is not None:
            if self.id_encoder_ is not None:
                X = self.id_encoder_.transform(X)
            X = self.frame_preprocessor_.transform(X).to_numpy(np.float32)
        else:
            X = _to_numpy_2d(X)
        if X.shape[1] != self.n_features_in_:
            raise ValueError(f"X has {X.shape[1]} features, the context has {self.n_features_in_}")
        return X

    # ------------------------------------------------------------------ sklearn API
    def fit(self, X, y):
        from synthefy_nori_b200.inference.large_context import resolve_policy
        from synthefy_nori_b200.inference.memory_policy import MemoryPolicy

        self.device_ = _as_device(self.device)
        MemoryPolicy.coerce(self.memory_policy)  # validate early (the reference validates in fit)
        if self.large_context_policy is not None:
            resolve_policy(self.large_context_policy)
        Xn = self._fit_features(X)
        Y = np.asarray(y, dtype=np.float64)
        if Y.ndim == 2 and Y.shape[1] == 1:
            Y = Y[:, 0]
        if Xn.shape[0] != Y.shape[0]:
            raise ValueError("X and y have different row counts")
        if Xn.shape[0] < 2:
            raise ValueError("need at least 2 context rows")
        if not np.all(np.isfinite(Y)):
            raise ValueError("y must be finite")
        self.X_train_ = Xn
        self.n_features_in_ = Xn.shape[1]
        self.context_ = self.context_yj_ = None
        self.predictor_ = None
        self.large_context_state_ = {}
        self.multi_target_ = None
        if Y.ndim == 2:
            from synthefy_nori_b200.multi_target_fit import MultiTargetFit

            self.y_train_ = Y
            self.multi_target_ = MultiTargetFit(self, Y)
            return self
        self.y_train_ = Y
        self.y_mean_ = float(Y.mean())
        std = float(Y.std())
        self.y_std_ = std if std > 0 else 1.0
        return self

    def _clone_for(self, X, y):
        """A fitted single-target regressor on (X, y) sharing this one's model."""
        params = self.get_params()
        params.update(discretize=None, categorical_levels=None, large_context_policy=None, augmentations=())
        child = type(self)(**params)
        child._model_obj = self._load_model()
        child.device_ = self.device_
        child.X_train_ = np.asarray(X, np.float32)
        child.n_features_in_ = child.X_train_.shape[1]
        child.categorical_features_ = list(getattr(self, "categorical_features_", []))
        child.frame_preprocessor_ = None
        child.context_ = child.context_yj_ = child.predictor_ = None
        child.multi_target_ = None
        child.large_context_state_ = {}
        yy = np.asarray(y, np.float64)
        child.y_train_, child.y_mean_ = yy, float(yy.mean())
        s = float(yy.std())
        child.y_std_ = s if s > 0 else 1.0
        return child

    def _context(self, yj: bool = False):
        attr = "context_yj_" if yj else "context_"
        if getattr(self, attr, None) is None:
            pred = self._get_predictor()
            if yj:
                yn = self.yj_.transform(self.y_train_.reshape(-1, 1)).ravel()
            else:
                yn = (self.y_train_ - self.y_mean_) / self.y_std_
            setattr(self, attr, pred.fit_context(self.X_train_, yn.astype(np.float32),
                                                 categorical=self.categorical_features_))
        return getattr(self, attr)

    def _raw(self, X: np.ndarray) -> torch.Tensor:
        while True:  # out of memory: escalate down the rung ladder and retry
            try:
                return self._get_predictor().predict_raw(self._context(), X)
            except torch.cuda.OutOfMemoryError as exc:
                if not self._escalate_memory(exc):
                    raise

    def _distribution(self, X: np.ndarray) -> dict:
        pred = self._get_predictor()
        raw = self._raw(X)
        mean, _, srt = pred.decode(raw, levels=[0.5], return_sorted=True)
        scale, shift = self.y_std_, self.y_mean_
        return {"quantiles": (srt * scale + shift).cpu().numpy().astype(np.float64),
                "taus": pred.taus.cpu().numpy().astype(np.float64),
                "mean": (mean * scale + shift).cpu().numpy().astype(np.float64)}

    def predict_distribution(self, X) -> dict:
        """Full predictive distribution: ascending quantiles ``[n, K]`` (y units), their
        levels ``taus [K]`` and the distribution mean ``[n]``."""
        self._check_fitted()
        if self._large_context_active():
            from synthefy_nori_b200.inference.large_context import LargeContextUnsupportedOutputError

            raise LargeContextUnsupportedOutputError(
                "a large-context policy returns point predictions only; use output_type='mean'/'median'/'mode' "
                "or raise large_context_threshold")
        return self._distribution(self._query_features(X))

    def _check_fitted(self):
        if not hasattr(self, "X_train_"):
            raise RuntimeError("call fit() before predict()")

    def _large_context_active(self) -> bool:
        from synthefy_nori_b200.inference.large_context import large_context_applies

        return large_context_applies(len(self.X_train_), self.large_context_policy, self.large_context_threshold)

    def _point(self, X: np.ndarray, mode: str) -> np.ndarray:
        """Point predictions with a collapse strategy, plus the Yeo-Johnson second pass
        for heavily skewed targets."""
        pred = self._get_predictor()
        point, _, _ = pred.decode(self._raw(X), collapse_mode=mode)
        base = (point.double() * self.y_std_ + self.y_mean_).cpu().numpy()
        if "yj" not in tuple(self.augmentations or ()) or len(self.y_train_) < 10:
            return base
        from scipy import stats

        skew = float(stats.skew(self.y_train_, bias=False))
        if not np.isfinite(skew) or abs(skew) < self.yj_skew_threshold:
            return base
        from sklearn.preprocessing import PowerTransformer

        if getattr(self, "yj_", None) is None:
            with warnings.catch_warnings():
                warnings.simplefilter("ignore")
                self.yj_ = PowerTransformer(method="yeo-johnson", standardize=True).fit(self.y_train_.reshape(-1, 1))
        raw = pred.predict_raw(self._context(yj=True), X)
        p_yj, _, _ = pred.decode(raw, collapse_mode=mode)
        p_yj = p_yj.double().cpu().numpy()
        ty = self.yj_.transform(self.y_train_.reshape(-1, 1)).ravel()
        span = (ty.max() - ty.min()) * 3.0 + 1e-6
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            inv = self.yj_.inverse_transform(np.clip(p_yj, ty.min() - span, ty.max() + span).reshape(-1, 1)).ravel()
        inv = np.where(np.isfinite(inv), inv, base)
        return 0.5 * (base + inv)

    def _large_context_point(self, X: np.ndarray, mode: str) -> np.ndarray:
        from synthefy_nori_b200.inference.large_context import run_policy

        def predict_fn(Xc, yc, Xq):
            return self._clone_for(Xc, yc)._point(np.asarray(Xq, np.float32), mode)

        window = self.large_context_window or min(len(self.X_train_), 50_000)
        preds, report = run_policy(self.large_context_policy, self.X_train_, self.y_train_, X, window=window,
                                   predict_fn=predict_fn, seed=self.random_state,
                                   train_cache=self.large_context_state_)
        self.large_context_report_ = report
        return preds

    def predict(self, X, *, output_type: str = "mean", quantiles: list[float] | None = None,
                discretize: str | None = None, categorical_levels=None, multi_target_prediction_policy=None):
        """``output_type``: ``"mean"`` (default, with ``quantile_collapse``), ``"median"``,
        ``"mode"`` (the median for a quantile head), ``"quantiles"`` (returns
        ``(len(quantiles), n)``) or ``"full"`` (dict, see ``predict_distribution``);
        ``discretize=`` / ``categorical_levels=`` return labels on the target's lattice.
        Multi-target fits take ``"mean"`` or ``"samples"``."""
        self._check_fitted()
        if self.multi_target_ is not None:
            if discretize is not None or categorical_levels is not None:
                raise ValueError("discretize and categorical_levels are not supported for multi-target regression")
            return self.multi_target_.predict(self._query_features(X), output_type=output_type,
                                              quantiles=quantiles, policy_override=multi_target_prediction_policy)
        X = self._query_features(X)
        discretize = self.discretize if discretize is None else discretize
        levels = self.categorical_levels if categorical_levels is None else categorical_levels
        if discretize is not None or levels is not None:
            if output_type != "mean" or quantiles is not None:
                raise ValueError("discretize=/categorical_levels= return labels; use them with output_type='mean'")
            return self._predict_categorical(X, discretize, levels)
        if output_type in ("quantiles", "full"):
            if self._large_context_active():
                return self.predict_distribution(X)  # raises the unsupported-output error
            if output_type == "full":
                return self._distribution(X)
            if not quantiles:
                raise ValueError("output_type='quantiles' needs quantiles=[...] in (0, 1)")
            if any(not (0.0 < float(t) < 1.0) for t in quantiles):
                raise ValueError("quantile levels must lie in (0, 1)")
            pred = self._get_predictor()
            _, q, _ = pred.decode(self._raw(X), levels=quantiles)
            return (q.double() * self.y_std_ + self.y_mean_).T.cpu().numpy()
        if output_type not in ("mean", "median", "mode"):
            raise ValueError(f"unknown output_type {output_type!r}; expected mean, median, mode, quantiles or full")
        if quantiles is not None:
            raise ValueError("quantiles= is only valid with output_type='quantiles'")
        mode = self.quantile_collapse if output_type == "mean" else "median"
        if self._large_context_active():
            return self._large_context_point(X, mode)
        return self._point(X, mode)

    def _predict_categorical(self, X: np.ndarray, method: str | None, levels) -> np.ndarray:
        from synthefy_nori_b200.discretize import (CONTINUOUS_METHODS, DEFAULT_DISCRETIZE_METHOD, SNAP_METHODS,
                                                   discretize_predictions, target_levels)

        method = DEFAULT_DISCRETIZE_METHOD if method is None else method
        lv = target_levels(self.y_train_) if levels is None else np.asarray(levels, np.float64)
        if method in SNAP_METHODS or method == "prior-match":
            mode = "median" if method == "snap-median" else "mean"
            point = self._point(X, mode) if not self._large_context_active() else self._large_context_point(X, mode)
            return discretize_predictions(method, lv, point=point, y_train=self.y_train_)
        d = self.predict_distribution(X)
        out = discretize_predictions(method, lv, Q=d["quantiles"], taus=d["taus"])
        return out if method in CONTINUOUS_METHODS else out.astype(np.float64)

    def get_embeddings(self, X=None, *, data_source: str = "test") -> np.ndarray:
        """Final-layer target-token states ``[members, n_rows, embed_dim]`` of the query
        rows (``data_source="test"``) or of the context rows (``"train"``, X ignored)."""
        self._check_fitted()
        if self.multi_target_ is not None:
            raise NotImplementedError("get_embeddings is not defined for a multi-target fit")
        pred = self._get_predictor()
        if data_source == "train":
            yn = ((self.y_train_ - self.y_mean_) / self.y_std_).astype(np.float32)
            return pred.context_embeddings(self.X_train_, yn, categorical=self.categorical_features_).cpu().numpy()
        if data_source != "test":
            raise ValueError("data_source must be 'test' or 'train'")
        if X is None:
            raise ValueError("get_embeddings requires X for data_source='test'")
        return pred.predict_raw(self._context(), self._query_features(X), return_hidden=True).cpu().numpy()

    @property
    def memory_report_(self) -> dict:
        ctx = getattr(self, "context_", None)
        pol = getattr(self, "memory_policy_", None)
        rep = pol.describe() if pol is not None else {}
        pred = getattr(self, "predictor_", None)
        rep.update({
            "cache_bytes": ctx.nbytes() if ctx is not None else 0,
            "context_rows": int(self.X_train_.shape[0]) if hasattr(self, "X_train_") else 0,
            "context_store_hits": pred.store.hits if pred is not None and pred.store is not None else 0,
        })
        return rep


def infer(X_train, y_train, X_test, *, model: str = "nori-6m", output_type: str = "mean", quantiles=None, **kw):
    """One-shot ``fit`` + ``predict`` (reference ``api.py:1383``)."""
    pkw = {k: kw.pop(k) for k in ("discretize", "categorical_levels") if k in kw}
    return NoriRegressor(model=model, **kw).fit(X_train, y_train).predict(X_test, output_type=output_type,
                                                                         quantiles=quantiles, **pkw)


def predict(X_train, y_train, X_test, **kw):
    """Alias of :func:`infer` (reference ``api.py:1443``)."""
    return infer(X_train, y_train, X_test, **kw)
