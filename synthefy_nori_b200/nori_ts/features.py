"""Time features for tabular forecasting (reference
``libs/synthefy/src/synthefy/nori_ts/tsfeatures``: running index, calendar components with
sin/cos seasonalities, FFT-detected seasonal periods).

Frames are indexed by ``(item_id, timestamp)``.  Calendar indices are zero-based
(second of minute, minute of hour, hour of day, day of week, day of month - 1, day of year
- 1, ISO week - 1, month - 1).  Seasonal periods are found per series from the magnitude
spectrum of the linearly detrended, Hann-windowed, zero-padded history: local peaks above
5% of the largest magnitude, strongest first, rounded to whole steps, at most ``max_top_k``.
The spectra of all series are computed as one batched ``torch.fft.rfft``.
"""

from __future__ import annotations

import numpy as np
import pandas as pd
import torch

DEFAULT_SEASONALITIES = {"second_of_minute": [60], "minute_of_hour": [60], "hour_of_day": [24], "day_of_week": [7],
                         "day_of_month": [30.5], "day_of_year": [365], "week_of_year": [52], "month_of_year": [12]}


def _calendar_index(ts: pd.DatetimeIndex, name: str) -> np.ndarray:
    return {
        "second_of_minute": lambda: ts.second, "minute_of_hour": lambda: ts.minute, "hour_of_day": lambda: ts.hour,
        "day_of_week": lambda: ts.dayofweek, "day_of_month": lambda: ts.day - 1, "day_of_year": lambda: ts.dayofyear - 1,
        "week_of_year": lambda: ts.isocalendar().week.to_numpy().astype(np.int64) - 1,
        "month_of_year": lambda: ts.month - 1,
    }[name]().astype(np.int64) if name in DEFAULT_SEASONALITIES else None


class RunningIndexFeature:
    def __call__(self, df: pd.DataFrame) -> pd.DataFrame:
        df = df.copy()
        df["running_index"] = df.groupby(level="item_id", sort=False).cumcount()
        return df


class CalendarFeature:
    def __init__(self, components=None, seasonal_features=None):
        self.components = components or ["year"]
        self.seasonal_features = seasonal_features or DEFAULT_SEASONALITIES

    def __call__(self, df: pd.DataFrame) -> pd.DataFrame:
        df = df.copy()
        ts = pd.DatetimeIndex(df.index.get_level_values("timestamp"))
        for c in self.components:
            df[c] = getattr(ts, c)
        for name, periods in self.seasonal_features.items():
            idx = np.asarray(_calendar_index(ts, name))
            if periods is None:
                df[name] = idx
                continue
            for k, p in enumerate(periods):
                sfx = f"_{k}" if len(periods) > 1 else ""
                df[f"{name}_sin{sfx}"] = np.sin(2 * np.pi * idx / p)
                df[f"{name}_cos{sfx}"] = np.cos(2 * np.pi * idx / p)
        return df


def seasonal_periods(series: list[np.ndarray], max_top_k: int = 12, threshold: float = 0.05,
                     pad_factor: int = 2) -> list[list[float]]:
    """Dominant periods per series (see the module docstring), batched over series."""
    if not series:
        return []
    n_max = max(len(s) for s in series)
    L = max(8, int(2 ** np.ceil(np.log2(max(n_max, 2) * pad_factor))))
    X = torch.zeros(len(series), L, dtype=torch.float64)
    for i, s in enumerate(series):
        v = np.asarray(s, np.float64)
        v = np.where(np.isfinite(v), v, np.nanmean(v) if np.isfinite(v).any() else 0.0)
        n = len(v)
        if n < 4:
            continue
        t = np.arange(n)
        a, b = np.polyfit(t, v, 1)
        d = (v - (a * t + b)) * np.hanning(n)
        X[i, :n] = torch.from_numpy(d)
    mag = torch.fft.rfft(X, dim=1).abs()
    mag[:, 0] = 0.0
    out = []
    for i, s in enumerate(series):
        m = mag[i].numpy()
        if len(s) < 4 or m.max() <= 0:
            out.append([])
            continue
        peaks = np.flatnonzero((m[1:-1] > m[:-2]) & (m[1:-1] >= m[2:])) + 1
        peaks = peaks[m[peaks] >= threshold * m.max()]
        peaks = peaks[np.argsort(-m[peaks])]
        found = []
        for k in peaks:
            p = float(np.round(L / k))
            if 2 <= p <= len(s) and p not in found:
                found.append(p)
            if len(found) >= max_top_k:
                break
        out.append(found)
    return out


class AutoSeasonalFeature:
    def __init__(self, max_top_k: int = 12):
        self.max_top_k = max_top_k

    def __call__(self, df: pd.DataFrame, history_mask: np.ndarray | None = None) -> pd.DataFrame:
        pos = df.groupby(level="item_id", sort=False).cumcount().to_numpy()
        codes, uniq = pd.factorize(df.index.get_level_values("item_id"), sort=False)
        hist = np.ones(len(df), bool) if history_mask is None else history_mask
        tgt = df["target"].to_numpy(np.float64)
        periods = seasonal_periods([tgt[(codes == c) & hist] for c in range(len(uniq))], self.max_top_k)
        P = np.full((len(uniq), self.max_top_k), np.nan)
        for c, ps in enumerate(periods):
            P[c, : len(ps)] = ps
        per = P[codes]
        with np.errstate(divide="ignore", invalid="ignore"):
            ang = 2 * np.pi * pos[:, None] / per
        ok = np.isfinite(per)
        cols = {}
        for i in range(self.max_top_k):
            cols[f"sin_#{i}"] = np.where(ok[:, i], np.sin(ang[:, i]), 0.0)
            cols[f"cos_#{i}"] = np.where(ok[:, i], np.cos(ang[:, i]), 0.0)
        return pd.concat([df, pd.DataFrame(cols, index=df.index)], axis=1)


def default_features() -> list:
    return [RunningIndexFeature(), CalendarFeature(), AutoSeasonalFeature()]


class PeriodicSinCosineFeature:
    """``sin`` / ``cos`` of ``2 pi t / period`` for fixed periods, with ``t`` the row position
    in the frame (reference ``tsfeatures/basic_features.py:103-121``: columns
    ``sin_<suffix>`` / ``cos_<suffix>``, the suffix being the period or ``<name_suffix>_<i>``)."""

    def __init__(self, periods, name_suffix: str | None = None):
        self.raw_periods = list(periods)
        self.periods = [float(p) for p in periods]
        self.name_suffix = name_suffix

    def generate(self, df: pd.DataFrame) -> pd.DataFrame:
        if not self.periods:
            return df.copy()
        t = np.arange(len(df), dtype=np.float64)
        cols = {}
        for period, raw in zip(self.periods, self._labels()):
            ang = 2.0 * np.pi * t / period
            cols[f"sin_{raw}"], cols[f"cos_{raw}"] = np.sin(ang), np.cos(ang)
        return pd.concat([df, pd.DataFrame(cols, index=df.index)], axis=1)

    __call__ = generate

    def _labels(self):
        if self.name_suffix:
            return [f"{self.name_suffix}_{i}" for i in range(len(self.periods))]
        return [_period_label(p) for p in self.raw_periods]


def _period_label(p) -> str:
    """The period as the caller wrote it: ``7`` for ints, ``30.5`` for fractional periods."""
    return str(p)


def _lowess_trend(x: np.ndarray, frac: float = 0.1) -> np.ndarray:
    """Locally weighted linear regression of ``x`` on its index (Cleveland 1979): at every
    point a straight line is fitted to the ``ceil(frac n)`` nearest points with tricube
    weights ``(1 - (d / d_max)^3)^3``; one pass, no robustness iterations."""
    n = len(x)
    t = np.arange(n, dtype=np.float64)
    k = max(2, min(n, int(np.ceil(frac * n))))
    trend = np.empty(n)
    for i in range(n):
        lo = min(max(0, i - k // 2), n - k)
        idx = slice(lo, lo + k)
        d = np.abs(t[idx] - t[i])
        dmax = max(d.max(), 1e-12) * (1.0 + 1e-12)
        w = (1.0 - (d / dmax) ** 3) ** 3
        tw, xw = t[idx], x[idx]
        sw = w.sum()
        mt, mx = (w * tw).sum() / sw, (w * xw).sum() / sw
        var = (w * (tw - mt) ** 2).sum()
        slope = (w * (tw - mt) * (xw - mx)).sum() / var if var > 0 else 0.0
        trend[i] = mx + slope * (t[i] - mt)
    return trend


def detrend(x: np.ndarray, detrend_type: str) -> np.ndarray:
    """Remove a trend from a series (reference ``tsfeatures/auto_features.py:275-299``):
    ``first_diff`` (differences, first element repeated), ``linear`` (least-squares line),
    ``constant`` (the mean) or ``loess`` (a local-linear smoother over 10% of the points)."""
    x = np.asarray(x, dtype=np.float64)
    if detrend_type == "first_diff":
        return np.diff(x, prepend=x[:1])
    if detrend_type == "linear":
        t = np.arange(len(x), dtype=np.float64)
        A = np.stack((t, np.ones_like(t)), 1)
        coef, *_ = np.linalg.lstsq(A, x, rcond=None)
        return x - A @ coef
    if detrend_type == "constant":
        return x - x.mean()
    if detrend_type == "loess":
        return x - _lowess_trend(x, 0.1)
    raise ValueError(f"Invalid detrend method: {detrend_type}")


def split_time_series_to_X_y(df: pd.DataFrame, target_col: str = "target"):
    """(features, target) frames of a time-series frame."""
    return df.drop(columns=[target_col]), df[[target_col]]
