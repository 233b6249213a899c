"""Nori-TS: seasonal period detection, features, forecaster on a tiny model."""

import numpy as np
import pandas as pd

from synthefy_nori_b200.nori_ts import CalendarFeature, NoriTSForecaster, seasonal_periods


def test_seasonal_periods_detects_cycles():
    t = np.arange(400)
    p = seasonal_periods([np.sin(2 * np.pi * t / 24) + 0.5 * np.sin(2 * np.pi * t / 7) + 0.01 * t], max_top_k=3)[0]
    assert 24.0 in p[:2] and 7.0 in p[:3]


def test_calendar_feature():
    idx = pd.MultiIndex.from_product([["a"], pd.date_range("2024-01-01", periods=3, freq="h")],
                                     names=["item_id", "timestamp"])
    df = CalendarFeature()(pd.DataFrame({"target": [1.0, 2, 3]}, index=idx))
    np.testing.assert_allclose(df["hour_of_day_sin"], np.sin(2 * np.pi * np.arange(3) / 24))
    assert (df["year"] == 2024).all()


class _Client:
    """Stand-in regression client: quantiles of a ridge fit."""

    def predict(self, Xtr, ytr, Xte, output_type, quantiles):
        A = np.c_[Xtr, np.ones(len(Xtr))]
        w = np.linalg.lstsq(A, ytr, rcond=None)[0]
        m = np.c_[Xte, np.ones(len(Xte))] @ w
        return np.stack([m + (q - 0.5) for q in quantiles])


def _frames():
    ts = pd.date_range("2024-01-01", periods=120, freq="D")
    rows = []
    for item, amp in (("a", 1.0), ("b", 3.0)):
        for k, t in enumerate(ts):
            rows.append((item, t, amp * np.sin(2 * np.pi * k / 7) + 0.05 * k))
    df = pd.DataFrame(rows, columns=["item_id", "timestamp", "target"]).set_index(["item_id", "timestamp"])
    hist = df.groupby(level="item_id").head(100)
    fut = df.groupby(level="item_id").tail(20)
    return hist, fut


def test_forecaster_with_client():
    hist, fut = _frames()
    f = NoriTSForecaster(client=_Client(), quantiles=[0.9, 0.1])
    out = f.predict(hist, fut.drop(columns="target"))
    assert list(out.columns) == ["target", "0.1", "0.9"] and len(out) == 40
    assert (out["0.1"] <= out["target"]).all() and (out["target"] <= out["0.9"]).all()
    err = np.abs(out["target"].to_numpy() - fut["target"].to_numpy()).mean()
    assert err < 0.5


def test_forecaster_local_tiny_model():
    hist, fut = _frames()
    f = NoriTSForecaster(model="nori-tiny", weights="random", device="cpu", n_estimators=1, context_length=64)
    out = f.predict(hist, fut.drop(columns="target"))
    assert out.shape == (40, 10) and np.isfinite(out.to_numpy()).all()
