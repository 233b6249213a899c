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
    np.testing.assert_allclose(qs[1], med, rtol=1e-5, atol=1e-5)
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
