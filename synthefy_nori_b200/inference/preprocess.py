"""Per-member feature preprocessing for the inference ensemble, on the device.

Parity target: reference ``inference/preprocess.py`` (steps 482-1848) and the member
construction in ``inference/predictor.py:353-418``; the member configurations use the
reference's JSON schema (``configs/default_inference.json``: eight members, four with
quantile-uniform rebalancing plus original columns and SVD features, four with the
per-column adaptive transform; ``model_v3_inference.json``: four members), so a
reference inference config runs unchanged.

The reference runs these steps with NumPy / scikit-learn on the host.  Here every
step is a tensor transform on the device that already holds the table (the context and
query rows are on the GPU for the model anyway): column quantiles, the quantile map,
SVD projections (``torch.linalg.svd``), polynomial products, MAD clipping, row hashing
and the column permutations all run as batched tensor ops.  Only the adaptive
transform's per-column power-transform fits (a one-parameter maximum likelihood and a
normality statistic, ``scipy.stats``) run on the host, on at most 3,000 values per column.

Step order per member (reference predictor.py:378-416): HighDimFeatureSelector ->
MaxFeatureSubsampler -> PolynomialInteractionGenerator -> FilterValidFeatures ->
MADWinsorizer -> RebalanceFeatureDistribution -> CategoricalFeatureEncoder ->
FingerprintFeatureEncoder -> FeatureShuffler.  Every step is fitted on the context rows
only and then applied to context and query rows (inductive), except the high-dimensional
SVD, which (``fit_on_test=True``, the shipped default) also sees the query rows'
features.
"""

from __future__ import annotations

import copy
import os
import warnings

import numpy as np
import torch

from synthefy_nori_b200.inference.degradation import SvdFallbackWarning

_QU = {"quantile_uniform_all_data", "quantile_uniform_5", "quantile_uniform_10"}
_QN = {"quantile_norm_all_data", "quantile_norm_5", "quantile_norm_10"}

_MEMBER_QUANTILE = {
    "MaxFeatureSubsampler": {"max_features": 500},
    "PolynomialInteractionGenerator": {"max_interaction_features": 10},
    "CategoricalFeatureEncoder": {"encoding_strategy": "ordinal_strict_feature_shuffled"},
    "FeatureShuffler": {"mode": "shuffle"},
    "RebalanceFeatureDistribution": {"worker_tags": ["quantile_uniform_all_data"], "discrete_flag": False,
                                     "original_flag": True, "svd_tag": "svd"},
    "FingerprintFeatureEncoder": True,
    "HighDimFeatureSelector": {"strategy": "svd_all", "svd_components": 512, "n_features_threshold": 256,
                               "binary_threshold": 1.01, "svd_rows_per_component": 3, "fit_on_test": True},
}
_MEMBER_ADAPTIVE = copy.deepcopy(_MEMBER_QUANTILE)
_MEMBER_ADAPTIVE["RebalanceFeatureDistribution"] = {"worker_tags": ["adaptive"], "discrete_flag": False,
                                                    "original_flag": False, "svd_tag": None}
DEFAULT_INFERENCE_CONFIG = [copy.deepcopy(_MEMBER_QUANTILE) for _ in range(4)] + \
    [copy.deepcopy(_MEMBER_ADAPTIVE) for _ in range(4)]
_V3_PLAIN = {k: v for k, v in _MEMBER_QUANTILE.items() if k not in ("HighDimFeatureSelector", "MaxFeatureSubsampler")}
MODEL_V3_INFERENCE_CONFIG = [
    copy.deepcopy(_MEMBER_QUANTILE),
    dict(copy.deepcopy(_V3_PLAIN), RebalanceFeatureDistribution={"worker_tags": ["quantile_uniform_all_data"],
                                                                 "discrete_flag": False, "original_flag": False,
                                                                 "svd_tag": None}),
    copy.deepcopy(_MEMBER_ADAPTIVE),
    {k: v for k, v in _V3_PLAIN.items() if k != "RebalanceFeatureDistribution"},
]


def _gen(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def _nan_fill_mean(x: torch.Tensor, mean: torch.Tensor) -> torch.Tensor:
    return torch.where(torch.isfinite(x), x, mean.expand_as(x))


def _col_nanmean(x: torch.Tensor) -> torch.Tensor:
    fin = torch.isfinite(x)
    cnt = fin.sum(0).clamp_min(1)
    return torch.where(fin, x, torch.zeros_like(x)).sum(0, keepdim=True) / cnt


def _interp(x: torch.Tensor, xp: torch.Tensor, fp: torch.Tensor) -> torch.Tensor:
    """Column-wise ``np.interp``: ``x [N, F]``, ``xp`` / ``fp`` ``[Q, F]`` (xp ascending)."""
    xt = x.t().contiguous()
    xpt = xp.t().contiguous()
    fpt = fp.t().contiguous() if fp.dim() == 2 else fp.unsqueeze(0).expand_as(xpt)
    j = torch.searchsorted(xpt, xt, right=True).clamp(1, xpt.shape[1] - 1)
    x0, x1 = xpt.gather(1, j - 1), xpt.gather(1, j)
    f0, f1 = fpt.gather(1, j - 1), fpt.gather(1, j)
    den = x1 - x0
    w = torch.where(den > 0, (xt - x0) / torch.where(den > 0, den, torch.ones_like(den)), torch.zeros_like(den))
    y = f0 + w.clamp(0, 1) * (f1 - f0)
    y = torch.where(xt <= xpt[:, :1], fpt[:, :1].expand_as(y), y)
    y = torch.where(xt >= xpt[:, -1:], fpt[:, -1:].expand_as(y), y)
    return y.t()


class Step:
    def fit(self, x: torch.Tensor, cat: list[int], seed: int, y=None, x_test=None) -> list[int]:
        raise NotImplementedError

    def transform(self, x: torch.Tensor, is_test: bool = False) -> torch.Tensor:
        raise NotImplementedError


class QuantileMap:
    """Quantile transform to uniform (or normal) scores, fitted per column; the forward
    and reversed interpolations are averaged so tied values map to the middle of their
    level range; NaN stays NaN."""

    def __init__(self, n_quantiles: int, output: str = "uniform"):
        self.n_quantiles, self.output = n_quantiles, output

    def fit(self, x: torch.Tensor) -> "QuantileMap":
        nq = max(2, min(self.n_quantiles, x.shape[0]))
        self.refs_ = torch.linspace(0, 1, nq, device=x.device, dtype=torch.float64)
        xd = x.double()
        q = torch.nanquantile(xd, self.refs_, dim=0) if x.shape[0] > 0 else xd.new_zeros(nq, x.shape[1])
        self.q_ = torch.nan_to_num(torch.cummax(q, 0).values, nan=0.0)
        return self

    def transform(self, x: torch.Tensor) -> torch.Tensor:
        xd = x.double()
        fwd = _interp(xd, self.q_, self.refs_)
        bwd = -_interp(-xd, (-self.q_).flip(0), (-self.refs_).flip(0))
        u = 0.5 * (fwd + bwd)
        if self.output == "normal":
            u = torch.special.ndtri(u.clamp(1e-7, 1 - 1e-7))
        return torch.where(torch.isnan(x), x.double(), u).to(x.dtype)


class KernelDensityIntegral:
    """Kernel-density-integral transform per column (McCarter, "The Kernel Density Integral
    Transformation", TMLR 2023), restated here from the paper: the CDF of a Gaussian kernel
    density estimate of the (NaN-free, NaN -> column mean) context values,

        F(x) = mean_i Phi((x - x_i) / h),   h = alpha * std(x),

    rescaled so the column minimum maps to 0 and the maximum to 1. Small ``alpha`` tends
    to the quantile transform, large ``alpha`` to min-max scaling. F is evaluated on a grid
    of ``n_grid`` points over [min, max] (one batched tensor op for all columns) and
    interpolated; ``output="normal"`` applies the normal quantile function to the result.
    Reference worker tags: ``kdi_uni`` / ``kdi_norm`` / ``kdi_*_alpha_<a>`` /
    ``norm_and_kdi`` (``inference/preprocess.py:1104-1150`` of the reference)."""

    def __init__(self, alpha: float = 1.0, output: str = "uniform", n_grid: int = 1024, chunk: int = 4096):
        if output not in ("uniform", "normal"):
            raise ValueError(f"unknown KDI output distribution {output!r}")
        self.alpha, self.output, self.n_grid, self.chunk = float(alpha), output, int(n_grid), int(chunk)

    def fit(self, x: torch.Tensor) -> "KernelDensityIntegral":
        xd = x.double()
        mean = _col_nanmean(xd)
        xd = _nan_fill_mean(xd, mean)
        n, p = xd.shape
        lo = xd.min(0).values if n else xd.new_zeros(p)
        hi = xd.max(0).values if n else xd.new_ones(p)
        sd = xd.std(0, unbiased=True) if n > 1 else xd.new_zeros(p)
        h = (self.alpha * sd).clamp_min(1e-12)
        t = torch.linspace(0, 1, self.n_grid, device=x.device, dtype=torch.float64)
        grid = lo[None] + t[:, None] * (hi - lo)[None]  # [G, p]
        cdf = xd.new_zeros(self.n_grid, p)
        for i in range(0, n, self.chunk):  # mean of Phi over the context values, in row chunks
            z = (grid[:, None, :] - xd[None, i : i + self.chunk, :]) / h
            cdf += torch.special.ndtr(z).sum(1)
        cdf /= max(n, 1)
        span = cdf[-1] - cdf[0]
        u = (cdf - cdf[0]) / torch.where(span > 0, span, torch.ones_like(span))
        const = (hi - lo) <= 0
        self.grid_ = torch.where(const[None], lo[None] + t[:, None], grid)
        self.u_ = torch.where(const[None], torch.full_like(u, 0.5), torch.cummax(u, 0).values)
        self.mean_ = mean
        return self

    def transform(self, x: torch.Tensor) -> torch.Tensor:
        xd = _nan_fill_mean(x.double(), self.mean_)
        u = _interp(xd, self.grid_, self.u_)
        if self.output == "normal":
            u = torch.special.ndtri(u.clamp(1e-7, 1 - 1e-7))
        return u.to(x.dtype)


def _kdi_worker(tag: str) -> "KernelDensityIntegral | None":
    """The reference's KDI worker tags -> a transform (None for other tags)."""
    if tag in ("kdi_uni", "kdi_norm"):
        return KernelDensityIntegral(1.0, "uniform" if tag == "kdi_uni" else "normal")
    for prefix, out in (("kdi_uni_alpha_", "uniform"), ("kdi_norm_alpha_", "normal")):
        if tag.startswith(prefix):
            return KernelDensityIntegral(float(tag[len(prefix):]), out)
    return None


class _Union:
    """Columns of several fitted transforms side by side (FeatureUnion)."""

    def __init__(self, parts):
        self.parts = parts

    def transform(self, x: torch.Tensor) -> torch.Tensor:
        return torch.cat([w.transform(x) for w in self.parts], 1)


class HighDimFeatureSelector(Step):
    def __init__(self, strategy: str = "svd_all", top_k: int = 256, n_features_threshold: int = 128,
                 binary_threshold: float = 0.5, svd_components: int = 64, svd_rows_per_component: int = 1,
                 fit_on_test: bool = False, extratrees_n_estimators: int = 100, subsample_rows: int = 5000):
        if strategy not in ("corr", "mi", "extratrees", "svd_binary", "svd_all", "passthrough"):
            raise ValueError(f"unknown HighDimFeatureSelector strategy {strategy!r}")
        self.strategy, self.top_k = strategy, int(top_k)
        self.n_features_threshold, self.binary_threshold = int(n_features_threshold), float(binary_threshold)
        self.svd_components, self.svd_rows_per_component = int(svd_components), max(1, int(svd_rows_per_component))
        self.fit_on_test = bool(fit_on_test)
        self.extratrees_n_estimators, self.subsample_rows = int(extratrees_n_estimators), int(subsample_rows)

    @staticmethod
    def _binary(x: torch.Tensor) -> torch.Tensor:
        fin = torch.isfinite(x)
        return (((x == 0) | (x == 1)) | ~fin).all(0) & fin.any(0)

    def fit(self, x, cat, seed, y=None, x_test=None):
        n, p = x.shape
        binary = self._binary(x)
        frac = float(binary.float().mean()) if p else 0.0
        self.mode_ = "passthrough"
        if self.strategy == "passthrough" or (p <= self.n_features_threshold and frac < self.binary_threshold):
            return cat
        if self.strategy in ("corr", "mi", "extratrees"):
            if y is None:
                return cat
            k = min(self.top_k, p)
            yt = torch.as_tensor(np.asarray(y), dtype=torch.float64, device=x.device)
            xf = _nan_fill_mean(x.double(), _col_nanmean(x.double()))
            if self.strategy == "corr":
                xc, yc = xf - xf.mean(0), yt - yt.mean()
                score = (xc * yc[:, None]).sum(0).abs() / (xc.norm(dim=0) * yc.norm()).clamp_min(1e-12)
                score = score.cpu().numpy()
            else:
                from sklearn.ensemble import ExtraTreesRegressor
                from sklearn.feature_selection import mutual_info_regression

                rows = _gen(seed).permutation(n)[: self.subsample_rows]
                Xh, yh = xf[rows].cpu().numpy(), yt[rows].cpu().numpy()
                score = (mutual_info_regression(Xh, yh, random_state=seed) if self.strategy == "mi" else
                         ExtraTreesRegressor(self.extratrees_n_estimators, random_state=seed, n_jobs=-1)
                         .fit(Xh, yh).feature_importances_)
            self.keep_ = torch.as_tensor(np.sort(np.argsort(-np.nan_to_num(score, nan=-1.0), kind="stable")[:k]),
                                         device=x.device)
            self.mode_ = "select"
            keep = set(self.keep_.tolist())
            return [i for i, c in enumerate(self.keep_.tolist()) if c in cat and c in keep]
        cols = torch.arange(p, device=x.device) if self.strategy == "svd_all" else torch.nonzero(binary).flatten()
        if self.strategy == "svd_binary" and frac < self.binary_threshold or cols.numel() < 2:
            return cat
        fit_rows = torch.cat([x, x_test], 0) if (self.fit_on_test and x_test is not None) else x
        sub = fit_rows[:, cols].double()
        self.mean_ = _col_nanmean(sub)
        sub = _nan_fill_mean(sub, self.mean_)
        self.center_ = sub.mean(0, keepdim=True)
        rank = min(self.svd_components, cols.numel() - 1, sub.shape[0] - 1, n // self.svd_rows_per_component)
        if rank < 1:
            return cat
        try:
            _, _, vh = torch.linalg.svd(sub - self.center_, full_matrices=False)
        except Exception as exc:  # noqa: BLE001
            warnings.warn(f"HighDimFeatureSelector: SVD failed ({type(exc).__name__}); keeping the columns",
                          SvdFallbackWarning, stacklevel=2)
            return cat
        comp = vh[:rank]
        # deterministic signs: largest-magnitude loading positive
        sgn = torch.sign(comp.gather(1, comp.abs().argmax(1, keepdim=True)))
        self.components_ = (comp * torch.where(sgn == 0, torch.ones_like(sgn), sgn)).t().contiguous()
        self.cols_ = cols
        self.rest_ = torch.nonzero(~torch.isin(torch.arange(p, device=x.device), cols)).flatten()
        self.mode_ = "svd"
        rest = self.rest_.tolist()
        return [i for i, c in enumerate(rest) if c in cat]

    def transform(self, x, is_test=False):
        if self.mode_ == "passthrough":
            return x
        if self.mode_ == "select":
            return x[:, self.keep_]
        sub = _nan_fill_mean(x[:, self.cols_].double(), self.mean_)
        proj = ((sub - self.center_) @ self.components_).to(x.dtype)
        return torch.cat([x[:, self.rest_], proj], 1)


class MaxFeatureSubsampler(Step):
    def __init__(self, max_features: int = 500):
        if max_features <= 0:
            raise ValueError("max_features must be > 0")
        self.max_features = int(max_features)

    def fit(self, x, cat, seed, y=None, x_test=None):
        p = x.shape[1]
        idx = np.arange(p) if p <= self.max_features else np.sort(_gen(seed).choice(p, self.max_features, False))
        self.idx_ = torch.as_tensor(idx, device=x.device)
        pos = {int(o): i for i, o in enumerate(idx)}
        return sorted(pos[c] for c in cat if c in pos)

    def transform(self, x, is_test=False):
        return x[:, self.idx_]


class PolynomialInteractionGenerator(Step):
    """Columns scaled to unit variance, then ``max_interaction_features`` random distinct
    products ``x_a * x_b`` (a <= b) appended."""

    def __init__(self, max_interaction_features: int | None = None, disable_above_n_features: int | None = None,
                 random_generator=None):
        self.max_interactions = int(max_interaction_features) if max_interaction_features else 100
        self.disable_above = disable_above_n_features

    def fit(self, x, cat, seed, y=None, x_test=None):
        p = x.shape[1]
        self.disabled_ = x.numel() == 0 or (self.disable_above is not None and p > self.disable_above)
        if self.disabled_:
            return cat
        xd = x.double()
        fin = torch.isfinite(xd)
        m = _col_nanmean(xd)
        var = (torch.where(fin, xd - m, torch.zeros_like(xd)) ** 2).sum(0) / fin.sum(0).clamp_min(1)
        sd = var.sqrt()
        self.scale_ = torch.where(sd > 0, sd, torch.ones_like(sd)).to(x.dtype)
        count = min(self.max_interactions, p * (p + 1) // 2)
        rng = _gen(seed)
        pairs, used = [], set()
        while len(pairs) < count:
            a = int(rng.integers(p))
            free = [b for b in range(a, p) if (a, b) not in used]
            if not free:
                continue
            b = int(rng.choice(free))
            used.add((a, b))
            pairs.append((a, b))
        pr = torch.as_tensor(pairs, device=x.device).reshape(-1, 2)
        self.a_, self.b_ = pr[:, 0], pr[:, 1]
        return cat

    def transform(self, x, is_test=False):
        if self.disabled_:
            return x
        z = x / self.scale_
        return torch.cat([z, z[:, self.a_] * z[:, self.b_]], 1)


class FilterValidFeatures(Step):
    """Drops columns that are constant (or all-NaN) on the context rows, and columns that
    are all-NaN on either the context or the query rows."""

    def fit(self, x, cat, seed, y=None, x_test=None):
        same = ((x == x[:1]) | (torch.isnan(x) & torch.isnan(x[:1]))).all(0)
        valid = ~same & ~torch.isnan(x).all(0)
        if x_test is not None and x_test.shape[0]:
            valid &= ~torch.isnan(x_test).all(0)
        if not bool(valid.any()):
            raise ValueError("all features are constant on the context rows")
        self.valid_ = torch.nonzero(valid).flatten()
        keep = self.valid_.tolist()
        return [i for i, c in enumerate(keep) if c in cat]

    def transform(self, x, is_test=False):
        return x[:, self.valid_]


class MADWinsorizer(Step):
    """Clip each non-categorical column at median +- n_mad * MAD of the context rows
    (plus a hard +-1e4 bound); ``soft_log_clip`` compresses the excess logarithmically."""

    def __init__(self, n_mad: float = 6.0, skip_categorical: bool = True, soft_log_clip: bool = False):
        self.n_mad, self.skip_categorical, self.soft = float(n_mad), bool(skip_categorical), bool(soft_log_clip)

    def fit(self, x, cat, seed, y=None, x_test=None):
        xd = x.double()
        med = torch.nanmedian(xd, 0).values
        mad = torch.nanmedian((xd - med).abs(), 0).values
        lo, hi = med - self.n_mad * mad, med + self.n_mad * mad
        active = torch.isfinite(mad) & (mad > 0)
        if self.skip_categorical and cat:
            active[torch.as_tensor(cat, device=x.device)] = False
        self.lo_ = torch.where(active, lo, torch.full_like(lo, -1e4)).clamp_min(-1e4).to(x.dtype)
        self.hi_ = torch.where(active, hi, torch.full_like(hi, 1e4)).clamp_max(1e4).to(x.dtype)
        return cat

    def transform(self, x, is_test=False):
        if not self.soft:
            return torch.where(torch.isnan(x), x, torch.minimum(torch.maximum(x, self.lo_), self.hi_))
        up = self.hi_ + torch.log1p((x - self.hi_).clamp_min(0))
        dn = self.lo_ - torch.log1p((self.lo_ - x).clamp_min(0))
        return torch.where(x > self.hi_, up, torch.where(x < self.lo_, dn, x))


class AdaptiveColumns:
    """Per-column transform chosen by the column's distribution on the context rows:
    < 10 distinct values: identity; non-negative with Fisher-Pearson skew > 5: log1p and
    standardise; |3 (mean - median) / std| > 1.1: exp for [0, 1] data, Box-Cox (positive)
    or Yeo-Johnson otherwise, then standardise; Shapiro-Wilk W > 0.95 on the first 3,000
    values: identity; otherwise a quantile map to normal scores."""

    def __init__(self, n_quantiles: int = 100, seed: int = 0):
        self.n_quantiles, self.seed = n_quantiles, seed

    def fit(self, x: torch.Tensor) -> "AdaptiveColumns":
        from scipy import stats

        X = x.double().cpu().numpy()
        self.kind_, self.param_ = [], []
        self.qmap_ = QuantileMap(self.n_quantiles, "normal").fit(x)
        for j in range(X.shape[1]):
            c = X[:, j]
            c = c[np.isfinite(c)]
            kind, par = "identity", None
            if len(c) >= 3 and len(np.unique(c)) >= 10:
                sd = c.std()
                mn, mx = c.min(), c.max()
                skew = 0.0 if sd < 1e-8 else float(np.clip(3.0 * (c.mean() - np.median(c)) / sd, -3, 3))
                fp = float(stats.skew(c, bias=False)) if mn >= 0 and sd > 1e-8 else 0.0
                if mn >= 0 and fp > 5.0:
                    t = np.log1p(c)
                    kind, par = "log1p", (t.mean(), t.std() or 1.0)
                elif abs(skew) > 1.1:
                    if mn >= 0 and mx <= 1.0:
                        kind = "exp"
                    elif mn > 0:
                        t, lam = stats.boxcox(c)
                        kind, par = "boxcox", (lam, t.mean(), t.std() or 1.0)
                    else:
                        t, lam = stats.yeojohnson(c)
                        kind, par = "yeojohnson", (lam, t.mean(), t.std() or 1.0)
                else:
                    w = stats.shapiro(c[:3000]).statistic if len(c) >= 3 else 1.0
                    kind = "identity" if w > 0.95 else "quantile"
            self.kind_.append(kind)
            self.param_.append(par)
        return self

    def transform(self, x: torch.Tensor) -> torch.Tensor:
        xd = x.double()
        out = xd.clone()
        q = None
        for j, (kind, par) in enumerate(zip(self.kind_, self.param_)):
            c = xd[:, j]
            if kind == "exp":
                out[:, j] = torch.exp(c)
            elif kind == "log1p":
                out[:, j] = (torch.log1p(c.clamp_min(-1 + 1e-12)) - par[0]) / par[1]
            elif kind == "boxcox":
                lam, mu, sd = par
                cc = c.clamp_min(1e-12)
                t = torch.log(cc) if abs(lam) < 1e-12 else (cc ** lam - 1) / lam
                out[:, j] = (t - mu) / sd
            elif kind == "yeojohnson":
                lam, mu, sd = par
                pos = c >= 0
                tp = torch.log1p(c.clamp_min(0)) if abs(lam) < 1e-12 else ((c.clamp_min(0) + 1) ** lam - 1) / lam
                cn = (-c).clamp_min(0)
                tn = -torch.log1p(cn) if abs(lam - 2) < 1e-12 else -((cn + 1) ** (2 - lam) - 1) / (2 - lam)
                out[:, j] = (torch.where(pos, tp, tn) - mu) / sd
            elif kind == "quantile":
                if q is None:
                    q = self.qmap_.transform(x).double()
                out[:, j] = q[:, j]
        return torch.where(torch.isnan(xd), xd, out).to(x.dtype)


class RebalanceFeatureDistribution(Step):
    def __init__(self, worker_tags=None, discrete_flag: bool = False, original_flag: bool = False,
                 svd_tag: str | None = None):
        self.worker_tags = list(worker_tags) if worker_tags is not None else ["quantile"]
        self.discrete_flag, self.original_flag, self.svd_tag = bool(discrete_flag), bool(original_flag), svd_tag

    def fit(self, x, cat, seed, y=None, x_test=None):
        n, p = x.shape
        dev = x.device
        cont = [i for i in range(p) if i not in cat]
        if self.original_flag:
            self.trans_ = cat + cont if self.discrete_flag else cont
            self.pass_ = list(range(p))
            new_cat = list(cat)
        elif self.discrete_flag:
            self.trans_, self.pass_, new_cat = cat + cont, [], []
        else:
            self.trans_, self.pass_, new_cat = cont, list(cat), list(range(len(cat)))
        self.workers_ = []
        xt = x[:, self.trans_] if self.trans_ else x[:, :0]
        for tag in self.worker_tags:
            if tag in _QU or tag in _QN or tag == "quantile":
                div = 10 if tag.endswith("_10") else 5
                w = QuantileMap(max(n // div, 2), "normal" if tag in _QN else "uniform").fit(xt)
            elif tag == "adaptive":
                w = AdaptiveColumns(max(n // 10, 2), seed).fit(xt)
            elif tag in ("robust", "squash"):
                med = torch.nanmedian(xt.double(), 0).values
                qs = torch.nanquantile(xt.double(), torch.tensor([0.25, 0.75], device=dev, dtype=torch.float64), 0)
                iqr = (qs[1] - qs[0]) / 1.3489795003921634  # unit variance for a normal column
                w = ("affine", med, torch.where(iqr > 0, iqr, torch.ones_like(iqr)))
            elif tag is None:
                w = None
            elif tag == "norm_and_kdi":
                w = _Union([QuantileMap(max(n // 10, 2), "normal").fit(xt),
                            KernelDensityIntegral(1.0, "uniform").fit(xt)])
            elif _kdi_worker(tag) is not None:
                w = _kdi_worker(tag).fit(xt)
            else:
                raise ValueError(f"worker tag {tag!r} is not provided by this build")
            self.workers_.append(w)
        self.svd_ = None
        if self.svd_tag == "svd" and p >= 2:
            k = max(1, min(n // 10 + 1, p // 2))
            xs = x.double()
            self.svd_mean_ = _col_nanmean(xs)
            xs = _nan_fill_mean(xs, self.svd_mean_)
            var = xs.pow(2).mean(0, keepdim=True)
            self.svd_scale_ = torch.where(var > 0, var.sqrt(), torch.ones_like(var))
            _, _, vh = torch.linalg.svd(xs / self.svd_scale_, full_matrices=False)
            comp = vh[:k]
            sgn = torch.sign(comp.gather(1, comp.abs().argmax(1, keepdim=True)))
            self.svd_ = (comp * torch.where(sgn == 0, torch.ones_like(sgn), sgn)).t().contiguous()
        return new_cat

    def transform(self, x, is_test=False):
        parts = [x[:, self.pass_]] if self.pass_ else []
        xt = x[:, self.trans_] if self.trans_ else x[:, :0]
        for w in self.workers_:
            if w is None:
                parts.append(xt)
            elif isinstance(w, tuple):
                parts.append(((xt.double() - w[1]) / w[2]).to(x.dtype))
            else:
                parts.append(w.transform(xt))
        out = torch.cat(parts, 1) if parts else x[:, :0]
        if self.svd_ is not None:
            xs = _nan_fill_mean(x.double(), self.svd_mean_) / self.svd_scale_
            out = torch.cat([out, (xs @ self.svd_).to(x.dtype)], 1)
        return out


class CategoricalFeatureEncoder(Step):
    """Ordinal codes (sorted context levels; unseen -> NaN) for the categorical columns,
    moved to the front; ``*_shuffled`` permutes each column's codes with the member seed;
    the ``*feature_shuffled`` strategies only encode columns whose rarest level occurs at
    least 10 times (``strict``: and with fewer than n/10 distinct values); other columns
    stay numeric.  ``numeric`` / ``none`` pass through."""

    def __init__(self, encoding_strategy: str | None = "ordinal"):
        if encoding_strategy not in ("ordinal", "ordinal_strict_feature_shuffled", "ordinal_shuffled", "onehot",
                                     "numeric", "none", None):
            raise ValueError(f"unknown categorical encoding {encoding_strategy!r}")
        self.encoding_strategy = encoding_strategy

    def fit(self, x, cat, seed, y=None, x_test=None):
        s = self.encoding_strategy
        self.order_ = None
        if s in (None, "none", "numeric") or not cat:
            return cat
        if s == "onehot":
            s = "ordinal"  # one-hot groups of two features would break per-group tokens; encode ordinally
        cols = list(cat)
        if "feature_shuffled" in s:
            keep = []
            for c in cols:
                _, counts = torch.unique(x[:, c], return_counts=True)  # NaN counts as its own value
                ok = counts.numel() > 0 and int(counts.min()) >= 10
                if "strict" in s:
                    ok = ok and counts.numel() < x.shape[0] // 10
                if ok:
                    keep.append(c)
            cols = keep
        p = x.shape[1]
        self.order_ = torch.as_tensor(cols + [i for i in range(p) if i not in cols], device=x.device)
        self.levels_ = [torch.unique(x[:, c][~torch.isnan(x[:, c])]) for c in cols]
        rng = _gen(seed)
        self.perm_ = [torch.as_tensor(rng.permutation(len(lv)), device=x.device, dtype=x.dtype)
                      if s.endswith("_shuffled") else None for lv in self.levels_]
        return list(range(len(cols)))

    def transform(self, x, is_test=False):
        if self.order_ is None:
            return x
        out = x[:, self.order_].clone()
        for j, (lv, pm) in enumerate(zip(self.levels_, self.perm_)):
            v = out[:, j]
            if lv.numel() == 0:
                out[:, j] = float("nan")
                continue
            idx = torch.searchsorted(lv, torch.nan_to_num(v, nan=0.0)).clamp_max(lv.numel() - 1)
            hit = (lv[idx] == v) & ~torch.isnan(v)
            code = idx.to(x.dtype) if pm is None else pm[idx]
            out[:, j] = torch.where(hit, code, torch.full_like(v, float("nan")))
        return out


def _row_hash(x: torch.Tensor, salt: int) -> torch.Tensor:
    """64-bit multiply-xorshift mix of each row's float32 bit patterns -> [0, 1)."""
    bits = x.float().contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    h = torch.full((x.shape[0],), (salt * 0x9E3779B1 + 0x632BE5AB) & 0x7FFFFFFFFFFFFFFF, dtype=torch.int64,
                   device=x.device)
    for j in range(bits.shape[1]):
        h = h ^ bits[:, j]
        h = (h * 0x5BD1E995) & 0x7FFFFFFFFFFFFFFF
        h = h ^ (h >> 29)
    return (h & ((1 << 53) - 1)).double() / float(1 << 53)


class FingerprintFeatureEncoder(Step):
    """Appends a per-row hash column (salted by the member seed).  Among context rows,
    repeated rows get distinct values (the k-th repeat hashes ``row + k``); query rows
    use their plain hash."""

    def fit(self, x, cat, seed, y=None, x_test=None):
        self.salt_ = int(_gen(seed).integers(0, 65536))
        return cat

    def transform(self, x, is_test=False):
        xs = torch.nan_to_num(x.float(), nan=-7.77e30) + self.salt_
        h = _row_hash(xs, self.salt_)
        if not is_test and x.shape[0] > 1:
            _, inv, cnt = torch.unique(xs, dim=0, return_inverse=True, return_counts=True)
            if bool((cnt > 1).any()):
                order = torch.argsort(inv, stable=True)
                start = torch.cumsum(cnt, 0) - cnt
                rank = torch.empty_like(inv)
                rank[order] = torch.arange(inv.numel(), device=x.device) - start[inv[order]]
                dup = rank > 0
                if bool(dup.any()):
                    h[dup] = _row_hash(xs[dup] + rank[dup, None].float(), self.salt_)
        return torch.cat([x, h.to(x.dtype).unsqueeze(1)], 1)


class FeatureShuffler(Step):
    def __init__(self, mode: str | None = "shuffle", offset: int = 0):
        if mode not in ("rotate", "shuffle", "latin", None):
            raise ValueError(f"unsupported reordering mode {mode!r}")
        self.mode, self.offset = mode, int(offset)

    def fit(self, x, cat, seed, y=None, x_test=None):
        p = x.shape[1]
        idx = np.arange(p)
        if self.mode == "rotate":
            idx = np.roll(idx, self.offset)
        elif self.mode == "shuffle":
            idx = _gen(seed).permutation(p)
        elif self.mode == "latin":
            idx = np.roll(_gen(seed).permutation(p), self.offset)
        self.idx_ = torch.as_tensor(idx, device=x.device)
        iscat = np.isin(np.arange(p), cat)
        return np.flatnonzero(iscat[idx]).tolist()

    def transform(self, x, is_test=False):
        return x[:, self.idx_]


def build_member(config: dict, offset: int = 0) -> list[Step]:
    """Steps of one ensemble member from a reference-schema config dict."""
    steps: list[Step] = []
    if "HighDimFeatureSelector" in config:
        steps.append(HighDimFeatureSelector(**config["HighDimFeatureSelector"]))
    if "MaxFeatureSubsampler" in config:
        steps.append(MaxFeatureSubsampler(**config["MaxFeatureSubsampler"]))
    if "PolynomialInteractionGenerator" in config:
        steps.append(PolynomialInteractionGenerator(**config["PolynomialInteractionGenerator"]))
    steps.append(FilterValidFeatures())
    if "MADWinsorizer" in config:
        steps.append(MADWinsorizer(**config["MADWinsorizer"]))
    if "RebalanceFeatureDistribution" in config:
        steps.append(RebalanceFeatureDistribution(**config["RebalanceFeatureDistribution"]))
    if "CategoricalFeatureEncoder" in config:
        steps.append(CategoricalFeatureEncoder(**config["CategoricalFeatureEncoder"]))
    if config.get("FingerprintFeatureEncoder", False):
        steps.append(FingerprintFeatureEncoder())
    if "FeatureShuffler" in config:
        steps.append(FeatureShuffler(**config["FeatureShuffler"], offset=offset))
    return steps


class MemberPipeline:
    """One ensemble member: fitted on the context rows (and, for the high-dimensional
    SVD, optionally the query rows' features), then applied to any query block."""

    def __init__(self, config: dict, seed: int, offset: int = 0):
        self.config, self.seed, self.steps = config, int(seed), build_member(config, offset)

    def fit_transform(self, x_ctx: torch.Tensor, y_ctx=None, x_test: torch.Tensor | None = None,
                      categorical: list[int] | None = None) -> torch.Tensor:
        cat = list(categorical or [])
        x, xt = x_ctx, x_test
        for i, s in enumerate(self.steps):
            cat = s.fit(x, cat, self.seed + i, y=y_ctx, x_test=xt)
            x = s.transform(x, is_test=False)
            if xt is not None:
                xt = s.transform(xt, is_test=True)
        self.categorical_ = cat
        self.n_out_ = x.shape[1]
        return x

    def transform(self, x: torch.Tensor) -> torch.Tensor:
        for s in self.steps:
            x = s.transform(x, is_test=True)
        return x


def member_seeds(n: int, seed: int) -> tuple[list[int], list[int]]:
    """Per-member seeds and distinct rotation offsets."""
    rng = _gen(seed)
    seeds = [int(v) for v in rng.integers(0, 2 ** 31 - 1, size=n)]
    offsets = [int(v) for v in rng.permutation(max(n, 1))[:n]]
    return seeds, offsets


def resolve_inference_config(config, model=None, n_estimators: int | None = None) -> list[dict]:
    """Explicit config list > ``"none"`` (identity members) > per-model default."""
    if config is None:
        base = MODEL_V3_INFERENCE_CONFIG if getattr(model, "two_phase_config", None) is not None \
            else DEFAULT_INFERENCE_CONFIG
    elif config == "none":
        base = [{}]
    elif isinstance(config, (str, os.PathLike)):  # a JSON file, or a bundled config's name
        from synthefy_nori_b200.configs import load_config

        base = list(load_config(os.fspath(config)))
    else:
        base = list(config)
    if n_estimators is not None and n_estimators > 0:
        base = [base[i % len(base)] for i in range(n_estimators)]
    return [copy.deepcopy(c) for c in base]


__all__ = [
    "DEFAULT_INFERENCE_CONFIG", "MODEL_V3_INFERENCE_CONFIG", "MemberPipeline", "build_member", "member_seeds",
    "resolve_inference_config", "QuantileMap", "HighDimFeatureSelector", "MaxFeatureSubsampler",
    "PolynomialInteractionGenerator", "FilterValidFeatures", "MADWinsorizer", "RebalanceFeatureDistribution",
    "CategoricalFeatureEncoder", "FingerprintFeatureEncoder", "FeatureShuffler", "AdaptiveColumns",
]
