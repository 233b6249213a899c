"""NoriRegressor / infer on CPU (random-init tiny model), quantile decode oracle."""

import numpy as np
import pytest
import torch

from synthefy_nori_b200.api import NoriRegressor, infer
from synthefy_nori_b200.inference.predictor import decode_torch


def _data(n=80, nq=20, f=5, seed=0):
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n + nq, f)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    w = rng.standard_normal(f)
    y = np.nan_to_num(X) @ w + 0.1 * rng.standard_normal(n + nq)
    return X[:n], y[:n], X[n:]


def test_regressor_outputs_and_clone():
    from sklearn.base import clone

    Xtr, ytr, Xte = _data()
    reg = NoriRegressor(model="nori-tiny", weights="random", device="cpu", n_estimators=2)
    reg.fit(Xtr, ytr)
    mean = reg.predict(Xte)
    assert mean.shape == (20,) and np.all(np.isfinite(mean))
    med = reg.predict(Xte, output_type="median")
    qs = reg.predict(Xte, output_type="quantiles", quantiles=[0.1, 0.5, 0.9])
    assert qs.shape == (3, 20)
    assert np.all(qs[0] <= qs[1] + 1e-6) and np.all(qs[1] <= qs[2] + 1e-6)
    # "median" is the bank's middle level (unsorted, as the reference's collapse);
    # quantiles interpolate the sorted bank
    raw = reg.predictor_.predict_raw(reg.context_, Xte)
    np.testing.assert_allclose(med, raw[:, 499].double().numpy() * reg.y_std_ + reg.y_mean_, rtol=1e-5, atol=1e-5)
    srt = raw.sort(-1).values
    np.testing.assert_allclose(qs[1], srt[:, 499].double().numpy() * reg.y_std_ + reg.y_mean_, rtol=1e-4, atol=1e-4)
    full = reg.predict(Xte, output_type="full")
    assert full["quantiles"].shape == (20, 999) and full["taus"].shape == (999,)
    np.testing.assert_allclose(full["mean"], mean, rtol=1e-5, atol=1e-5)
    # cache reuse: a second predict does not rebuild the context
    ctx = reg.context_
    reg.predict(Xte)
    assert reg.context_ is ctx
    c = clone(reg)
    assert c.get_params() == reg.get_params()
    with pytest.raises(ValueError):
        reg.predict(Xte[:, :3])


def test_infer_one_shot_and_int8_cache():
    Xtr, ytr, Xte = _data(seed=1)
    a = infer(Xtr, ytr, Xte, model="nori-tiny", weights="random", device="cpu")
    b = infer(Xtr, ytr, Xte, model="nori-tiny", weights="random", device="cpu", cache_dtype="int8")
    assert a.shape == b.shape == (20,)
    assert np.max(np.abs(a - b)) < 0.1 * (np.std(ytr) + 1e-6)


def test_decode_torch_matches_definition():
    torch.manual_seed(0)
    taus = torch.tensor([(i + 1) / 1000 for i in range(999)])
    raw = torch.randn(7, 999)
    mean, q, srt = decode_torch(raw, taus, torch.tensor([0.1, 0.5, 0.9]), return_sorted=True)
    s = raw.sort(-1).values
    assert torch.equal(srt, s)
    ref = taus[0] * s[:, 0] + (1 - taus[-1]) * s[:, -1] + ((s[:, 1:] + s[:, :-1]) / 2 * (taus[1:] - taus[:-1])).sum(-1)
    torch.testing.assert_close(mean, ref)
    torch.testing.assert_close(q[:, 1], s[:, 499])


def _reg(**kw):
    return NoriRegressor(model="nori-tiny", weights="random", device="cpu", n_estimators=2, **kw)


def test_discretize_and_collapse_strategies():
    Xtr, ytr, Xte = _data(seed=2)
    yd = np.round(ytr).clip(-2, 2)
    reg = _reg().fit(Xtr, yd)
    lv = np.unique(yd)
    for m in ("map-cell", "median-cell", "snap-mean", "snap-median", "prior-match"):
        out = reg.predict(Xte, discretize=m)
        assert out.shape == (20,) and set(np.unique(out)) <= set(lv)
    ev = reg.predict(Xte, discretize="expected-level")
    assert np.all((ev >= lv.min() - 1e-9) & (ev <= lv.max() + 1e-9))
    out = reg.predict(Xte, categorical_levels=[-3, -2, -1, 0, 1, 2, 3])
    assert set(np.unique(out)) <= {-3, -2, -1, 0, 1, 2, 3}
    with pytest.raises(ValueError):
        reg.predict(Xte, discretize="map-cell", output_type="median")
    for mode in ("median", "trimmed_mean", "huber_mean", "tail_aware", "qdist", "qdist_simple"):
        r = _reg(quantile_collapse=mode).fit(Xtr, ytr)
        assert np.all(np.isfinite(r.predict(Xte)))
    assert reg.predict(Xte, output_type="mode").shape == (20,)


def test_embeddings_dataframe_and_ids():
    import pandas as pd

    Xtr, ytr, Xte = _data(seed=3)
    reg = _reg().fit(Xtr, ytr)
    e = reg.get_embeddings(Xte)
    assert e.shape[0] == 2 and e.shape[1] == 20 and np.all(np.isfinite(e))
    et = reg.get_embeddings(data_source="train")
    assert et.shape[:2] == (2, 80)
    df = pd.DataFrame(Xtr, columns=[f"f{i}" for i in range(5)])
    df["shop"] = np.where(np.arange(80) % 3 == 0, "a", "b")
    df["kind"] = pd.Categorical(np.where(np.arange(80) % 2 == 0, "u", "v"))
    dq = pd.DataFrame(Xte, columns=[f"f{i}" for i in range(5)])
    dq["shop"] = "c"
    dq["kind"] = pd.Categorical(["u"] * 20)
    r = _reg(encode_id_cols=["shop"]).fit(df, ytr)
    assert r.predict(dq).shape == (20,)
    assert r.categorical_features_ == [6]  # "kind"; the ID column is numeric codes


@pytest.mark.parametrize("strategy", ["independent", "copula", "autoregressive"])
def test_multi_target(strategy):
    Xtr, ytr, Xte = _data(n=60, seed=4)
    Y = np.stack([ytr, 0.5 * ytr + np.sin(Xtr[:, 0].astype(np.float64).clip(-3, 3))], 1)
    Y = np.nan_to_num(Y)
    pol = {"n_draws": 12, "copula_cv": 2, "autoregressive_n_orders": 2}
    reg = _reg(multi_target_prediction_strategy=strategy, multi_target_prediction_policy=pol).fit(Xtr, Y)
    m = reg.predict(Xte)
    assert m.shape == (20, 2) and np.all(np.isfinite(m))
    s = reg.predict(Xte, output_type="samples")
    assert s.shape == (20, 12, 2) and np.all(np.isfinite(s))
    with pytest.raises(ValueError):
        reg.predict(Xte, output_type="quantiles", quantiles=[0.5])
    with pytest.raises(ValueError):
        reg.predict(Xte, multi_target_prediction_policy={"copula_cv": 3})


def test_large_context_policy_and_yj_pass():
    from synthefy_nori_b200.inference.large_context import LargeContextUnsupportedOutputError

    Xtr, ytr, Xte = _data(n=200, seed=5)
    reg = _reg(large_context_policy="cluster_route[groups=2]", large_context_threshold=100,
               large_context_window=64).fit(Xtr, ytr)
    p = reg.predict(Xte)
    assert p.shape == (20,) and reg.large_context_report_["nori_calls"] >= 1
    with pytest.raises(LargeContextUnsupportedOutputError):
        reg.predict(Xte, output_type="full")
    skewed = np.abs(ytr)
    skewed[0] = 1e6  # one extreme value: sample skew ~ sqrt(n) = 14 > 10
    r = _reg().fit(Xtr, skewed)
    a = r.predict(Xte)
    assert getattr(r, "yj_", None) is not None and np.all(np.isfinite(a))
    b = _reg(augmentations=()).fit(Xtr, skewed).predict(Xte)
    assert not np.allclose(a, b)
