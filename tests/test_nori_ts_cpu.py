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


def test_periodic_features_detrend_and_split():
    import pytest
    import numpy as np
    import pandas as pd

    from synthefy_nori_b200.nori_ts import PeriodicSinCosineFeature, detrend, split_time_series_to_X_y

    df = pd.DataFrame({"target": np.arange(14.0), "x": 1.0})
    out = PeriodicSinCosineFeature([7, 30.5]).generate(df)
    assert out.columns.tolist() == ["target", "x", "sin_7", "cos_7", "sin_30.5", "cos_30.5"]
    np.testing.assert_allclose(out["sin_7"].to_numpy()[[0, 7]], [0.0, 0.0], atol=1e-12)
    np.testing.assert_allclose(out["cos_7"].to_numpy()[7], 1.0)
    assert PeriodicSinCosineFeature([12], name_suffix="m").generate(df).columns[-2:].tolist() == ["sin_m_0", "cos_m_0"]
    t = np.arange(200.0)
    x = 3.0 * t + 5.0 + np.sin(t)
    np.testing.assert_allclose(detrend(x, "linear"), np.sin(t) - np.polyval(np.polyfit(t, np.sin(t), 1), t),
                               atol=1e-8)
    assert detrend(x, "first_diff")[0] == 0.0 and np.allclose(detrend(x, "first_diff")[1:], np.diff(x))
    assert abs(detrend(x, "constant").mean()) < 1e-9
    # a straight line is its own local-linear trend
    assert np.abs(detrend(3.0 * t + 1.0, "loess")).max() < 1e-9
    # loess removes a slow trend but keeps a fast oscillation
    slow = np.sin(t / 60.0) * 10 + np.sin(t * 2.5)
    assert np.corrcoef(detrend(slow, "loess"), np.sin(t * 2.5))[0, 1] > 0.9
    with pytest.raises(ValueError):
        detrend(x, "spline")
    X, y = split_time_series_to_X_y(df)
    assert X.columns.tolist() == ["x"] and y.columns.tolist() == ["target"]
