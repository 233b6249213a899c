"""CPU tests: decode strategies, discretize, entity IDs, pricing, DataFrame featurizer,
multi-target helpers, per-member preprocessing and large-context policies.  Where the
reference package is installed, its functions are the oracle."""

import warnings

import numpy as np
import pandas as pd
import pytest
import torch

from synthefy_nori_b200 import discretize as dz
from synthefy_nori_b200.inference import decode
from synthefy_nori_b200.inference import large_context as lc
from synthefy_nori_b200.inference import preprocess as pp
from synthefy_nori_b200.multi_target import (GaussianCopula, build_target_orders, cdf_from_quantile_bank,
                                             quantiles_from_levels)

TAUS = torch.tensor([(i + 1) / 1000 for i in range(999)], dtype=torch.float64)


def _bank(n=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    base = torch.randn(n, 1, generator=g, dtype=torch.float64)
    spread = torch.rand(n, 1, generator=g, dtype=torch.float64) + 0.1
    q = base + spread * torch.special.ndtri(TAUS)[None] + 0.01 * torch.randn(n, 999, generator=g, dtype=torch.float64)
    q[0] = q[0] ** 3  # a skewed row
    return q


@pytest.mark.parametrize("mode", decode.COLLAPSE_MODES)
def test_collapse_modes_match_reference(mode, reference_pkg):
    from synthefy_nori.inference.predictor import NoriPredictor as RefPredictor

    class _Ref(RefPredictor):
        regression_quantiles = tuple(TAUS.tolist())

    q = _bank().float()
    ref = _Ref.__new__(_Ref)
    ref.quantile_collapse = mode
    want = ref._apply_quantile_collapse(q).double()
    got = decode.collapse(q, TAUS.float(), mode).double()
    torch.testing.assert_close(got, want, rtol=2e-5, atol=2e-5)


def test_collapse_definitions_without_reference():
    q = _bank().double()
    qs = q.sort(-1).values
    m = decode.collapse(q, TAUS, "mean")
    ref = TAUS[0] * qs[:, 0] + (1 - TAUS[-1]) * qs[:, -1] + ((qs[:, 1:] + qs[:, :-1]) / 2 * TAUS.diff()).sum(-1)
    torch.testing.assert_close(m.double(), ref, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(decode.collapse(q, TAUS, "median").double(), q[:, 499].float().double())
    tails = decode.quantile_mean(q, TAUS, tails=True)
    assert torch.all(torch.isfinite(tails))
    with pytest.raises(ValueError):
        decode.collapse(q, TAUS, "nope")


def test_bar_decode():
    logits = torch.randn(5, 100)
    b = decode.uniform_borders(100)
    c = 0.5 * (b[:-1] + b[1:])
    p = logits.softmax(-1)
    torch.testing.assert_close(decode.bar_decode(logits, b, "mean"), (p * c).sum(-1))
    torch.testing.assert_close(decode.bar_decode(logits, b, "mode"), c[p.argmax(-1)])


def test_discretize_against_reference(reference_pkg):
    import importlib

    rd = importlib.import_module("synthefy_nori.discretize")
    rng = np.random.default_rng(0)
    Q = np.sort(rng.normal(2.0, 1.0, (40, 999)), 1)
    Q[:5] = np.round(Q[:5])  # ties / flat stretches
    taus = TAUS.numpy()
    levels = np.array([0, 1, 2, 3, 5], float)
    np.testing.assert_allclose(dz.cell_masses(Q, taus, levels), rd.cell_masses(Q, taus, levels), atol=1e-12)
    point = rng.normal(2, 2, 40)
    point[3], point[4], point[5] = np.nan, np.inf, -np.inf
    ytr = rng.choice(levels, 100)
    for m in dz.DISCRETIZE_METHODS:
        a = dz.discretize_predictions(m, levels, point=point, Q=Q, taus=taus, y_train=ytr)
        b = rd.discretize_predictions(m, levels, point=point, Q=Q, taus=taus, y_train=ytr)
        np.testing.assert_allclose(a, b, atol=1e-12, equal_nan=True)


def test_discretize_semantics():
    levels = np.array([1.0, 2.0, 3.0])
    np.testing.assert_array_equal(dz.snap_to_levels([1.5, 2.49, np.inf, -np.inf], levels), [2, 2, 3, 1])
    assert np.isnan(dz.snap_to_levels([np.nan], levels)[0])
    Q = np.tile(np.linspace(1.8, 2.2, 999), (2, 1))
    P = dz.cell_masses(Q, TAUS.numpy(), levels)
    np.testing.assert_allclose(P.sum(1), 1.0)
    assert np.all(dz.discretize_predictions("map-cell", levels, Q=Q, taus=TAUS.numpy()) == 2.0)
    out = dz.prior_match(np.arange(10.0), levels, [1, 1, 1, 1, 1, 2, 2, 2, 3, 3])
    np.testing.assert_array_equal(out, [1, 1, 1, 1, 1, 2, 2, 2, 3, 3])
    assert set(dz.DISCRETIZE_METHOD_DESCRIPTIONS) == set(dz.DISCRETIZE_METHODS)


def test_entity_ids_and_pricing():
    from synthefy_nori_b200.entity_ids import EntityIDPreprocessor
    from synthefy_nori_b200.pricing import billable_price

    tr = pd.DataFrame({"store": ["b", "a", "b", None], "x": [1.0, 2, 3, 4]})
    te = pd.DataFrame({"store": ["a", "z", None], "x": [1.0, 2, 3]})
    enc = EntityIDPreprocessor(["store"]).fit(tr)
    assert enc.transform(te)["store"].tolist() == [1, -1, -1]
    assert enc.transform(tr)["store"].tolist() == [0, 1, 0, -1]
    with pytest.raises(ValueError):
        EntityIDPreprocessor(["store", "store"])
    with pytest.raises(ValueError):
        EntityIDPreprocessor(["x"]).fit(tr)
    assert billable_price(0, 0) == pytest.approx(1.4 * 6.5 / 3600 * 0.6)
    assert billable_price(1000, 50) == pytest.approx(1.4 * 6.5 / 3600 * (3.0 + 6.0))


def test_dataframe_preprocessor():
    from synthefy_nori_b200.featurize import DataFramePreprocessor

    tr = pd.DataFrame({"a": [1.0, 2, 3, 4], "c": ["x", "y", "x", None], "t": ["red car", "blue bus", "red bus", "x"]})
    te = pd.DataFrame({"a": [5.0, 6], "c": ["y", "new"], "t": ["red", None]})
    pre = DataFramePreprocessor(text_columns=["t"], svd_dim=2)
    A = pre.fit_transform(tr)
    B = pre.transform(te)
    assert list(A.columns) == list(B.columns) and A.shape[1] == 4
    assert B["c"].tolist() == [1.0, 2.0]  # "y" -> 1, unseen -> other code 2
    assert np.isnan(A["c"].iloc[3])
    oh = DataFramePreprocessor(categorical_encoding="onehot").fit(tr[["a", "c"]])
    assert list(oh.get_feature_names_out()) == ["a", "c_x", "c_y", "c_nan"]
    with pytest.raises(ValueError):
        pre.transform(te[["a", "c"]])
    with pytest.raises(ValueError):
        DataFramePreprocessor(categorical_columns=None).fit(tr)


def test_multi_target_helpers(reference_pkg):
    import importlib

    rm = importlib.import_module("synthefy_nori.multi_target")
    rng = np.random.default_rng(0)
    Q = np.sort(rng.normal(0, 1, (30, 999)), 1)
    Q[:4, 100:300] = Q[:4, 100:101]  # flat stretch = atom
    y = rng.normal(0, 1.2, 30)
    y[0] = Q[0, 150]
    taus = TAUS.numpy()
    np.testing.assert_allclose(cdf_from_quantile_bank(Q, taus, y), rm.cdf_from_quantile_bank(Q, taus, y), atol=1e-12)
    U = rng.random((30, 7))
    np.testing.assert_allclose(quantiles_from_levels(Q, taus, U), rm.quantiles_from_levels(Q, taus, U), atol=1e-12)
    a = build_target_orders(3, 4, 0)
    assert len(a) == 4 and len({tuple(o) for o in a}) == 4 and list(a[0]) == [0, 1, 2]


def test_gaussian_copula_recovers_correlation():
    from scipy.stats import norm

    rng = np.random.default_rng(1)
    z = rng.multivariate_normal([0, 0], [[1, 0.8], [0.8, 1]], 4000)
    cop = GaussianCopula().fit(norm.cdf(z))
    assert abs(cop.corr_[0, 1] - 0.8) < 0.03
    s = cop.simulate(4000, rng)
    assert abs(np.corrcoef(norm.ppf(s), rowvar=False)[0, 1] - 0.8) < 0.05


def test_quantile_map_matches_sklearn():
    from sklearn.preprocessing import QuantileTransformer

    rng = np.random.default_rng(0)
    x = rng.standard_normal((600, 4))
    x[:, 1] = np.round(x[:, 1])
    t = rng.standard_normal((50, 4)) * 2
    t[:, 1] = np.round(t[:, 1])
    qt = QuantileTransformer(n_quantiles=120, subsample=600).fit(x)
    got = pp.QuantileMap(120).fit(torch.tensor(x)).transform(torch.tensor(t)).numpy()
    np.testing.assert_allclose(got, qt.transform(t), atol=1e-12)


def test_member_pipelines_are_inductive_and_consistent():
    torch.manual_seed(0)
    x = torch.randn(300, 12)
    x[:, 3] = torch.randint(0, 4, (300,)).float()
    x[::7, 2] = float("nan")
    xq = torch.randn(40, 12)
    for cfg in pp.DEFAULT_INFERENCE_CONFIG[::4] + pp.MODEL_V3_INFERENCE_CONFIG:
        m = pp.MemberPipeline(cfg, seed=5)
        a = m.fit_transform(x, None, None, categorical=[3])
        b = m.transform(x)
        # the fingerprint column differs only for repeated rows; everything else is inductive
        torch.testing.assert_close(a, b, equal_nan=True)
        c = m.transform(xq)
        assert c.shape[1] == a.shape[1] == m.n_out_
    wide = pp.MemberPipeline(pp.DEFAULT_INFERENCE_CONFIG[0], seed=1)
    out = wide.fit_transform(torch.randn(200, 400), None, torch.randn(20, 400))
    assert out.shape[1] < 400


def test_fingerprint_separates_repeated_context_rows():
    fp = pp.FingerprintFeatureEncoder()
    x = torch.tensor([[1.0, 2.0], [1.0, 2.0], [3.0, 4.0]])
    fp.fit(x, [], 0)
    a = fp.transform(x)[:, -1]
    assert a[0] != a[1]
    q = fp.transform(x, is_test=True)[:, -1]
    assert q[0] == q[1] == a[0]


def _fake_predict(Xc, yc, Xq):
    # nearest-neighbour regressor stand-in for the model
    d = ((Xq[:, None, :] - Xc[None, :, :]) ** 2).sum(-1)
    return yc[d.argmin(1)]


@pytest.mark.parametrize("spec", ["random", "target_rank", "target_rank[cap=100]", "cluster_route[groups=3]",
                                  "cluster_route_g4", "safeboost", "boost[patience=2]",
                                  ["random", "cluster_route[groups=2]"]])
def test_large_context_policies_run(spec):
    rng = np.random.default_rng(0)
    X = rng.standard_normal((1200, 3)).astype(np.float32)
    y = X[:, 0] * 2 + np.sin(X[:, 1])
    Xq = rng.standard_normal((64, 3)).astype(np.float32)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")  # boosting warns below its shard floor
        preds, rep = lc.run_policy(spec, X, y, Xq, window=300, predict_fn=_fake_predict, seed=0)
    assert preds.shape == (64,) and np.all(np.isfinite(preds)) and rep["nori_calls"] >= 1
    truth = Xq[:, 0] * 2 + np.sin(Xq[:, 1])
    assert lc.r2(truth, preds) > 0.5


def test_policy_registry_and_loader(tmp_path):
    f = tmp_path / "my_policy.py"
    f.write_text("import numpy as np\n"
                 "def first_rows(problem, rng, k=50):\n"
                 "    return problem.predict(np.arange(k))\n")
    name, fn = lc.resolve_policy(f"{f}:first_rows[k=20]")
    X = np.random.default_rng(0).standard_normal((100, 2)).astype(np.float32)
    p, rep = lc.run_policy(f"{f}:first_rows[k=20]", X, X[:, 0], X[:5], window=50, predict_fn=_fake_predict)
    assert p.shape == (5,)
    with pytest.raises(ValueError):
        lc.resolve_policy("does_not_exist")
    assert "cluster_route" in lc.registered_policies()
