"""Out-of-fold embeddings, the marginal / conditional imputers and NoriInterpreter on a
tiny random-weight model (CPU)."""

import numpy as np
import pytest


def _reg(**kw):
    from synthefy_nori_b200.api import NoriRegressor

    return NoriRegressor(model="nori-tiny", weights="random", device="cpu", n_estimators=1, **kw)


def test_oof_embeddings_match_manual_folds():
    from sklearn.model_selection import KFold

    from synthefy_nori_b200.embedding import NoriEmbedding

    rng = np.random.default_rng(0)
    X = rng.standard_normal((60, 4)).astype(np.float32)
    y = X[:, 0] - X[:, 1]
    emb = NoriEmbedding(n_fold=3, model=_reg(), shuffle=True, random_state=5)
    tr = emb.fit_transform(X, y)
    assert tr.shape[:2] == (1, 60)
    # row i of fold k equals embedding it as a query against the other folds
    ctx, held = next(KFold(3, shuffle=True, random_state=5).split(X))
    ref = _reg().fit(X[ctx], y[ctx]).get_embeddings(X[held], data_source="test")
    np.testing.assert_allclose(tr[:, held], ref, rtol=1e-4, atol=1e-5)
    # transform uses the full-data model
    full = _reg().fit(X, y).get_embeddings(X[:7], data_source="test")
    np.testing.assert_allclose(emb.transform(X[:7]), full, rtol=1e-4, atol=1e-5)
    with pytest.raises(ValueError):
        NoriEmbedding(n_fold=1, model=_reg()).fit(X, y)
    with pytest.raises(ValueError):
        NoriEmbedding(n_fold=2).fit(X, y)


def _linear(rows):
    rows = np.asarray(rows, np.float64)
    return 3 * rows[:, 0] - 2 * rows[:, 1] + 0.5 * rows[:, 2]


@pytest.mark.parametrize("imputer", ["baseline", "marginal", "conditional"])
def test_imputers_efficiency_and_linear_values(imputer):
    from synthefy_nori_b200.interpretability.shapley import ImputationExplainer

    rng = np.random.default_rng(1)
    bg = rng.standard_normal((200, 3))
    x = np.array([1.0, -1.0, 2.0])
    ex = ImputationExplainer(_linear, bg, index="SV", imputer=imputer, n_samples=200 if imputer == "marginal" else 25)
    iv = ex.explain(x, budget=64)
    phi = iv.values_array(3)
    # efficiency: the values add up to f(x) - value of the empty coalition
    assert abs(phi.sum() - (_linear(x[None])[0] - iv[()])) < 1e-9
    if imputer != "conditional":  # a linear model's interventional values are w_i (x_i - E[x_i])
        mu = bg.mean(0)
        np.testing.assert_allclose(phi, np.array([3, -2, 0.5]) * (x - mu), atol=1e-9)
    else:  # independent features: the nearest-neighbour conditional stays close to that
        assert np.sign(phi[0]) == 1 and np.sign(phi[1]) == 1


def test_interpreter_regression_and_binary():
    from synthefy_nori_b200.interpretability import NoriInterpreter

    rng = np.random.default_rng(2)
    X = rng.standard_normal((160, 20)).astype(np.float32)
    y = 2 * X[:, 3] + X[:, 7]
    it = NoriInterpreter("nori-tiny", regressor_kwargs=dict(weights="random", device="cpu", n_estimators=1),
                         rounds=40, n_repeats=1).fit(X, y)
    assert it.task_ == "regression" and it.reduced_
    assert len(it.feature_importances_) == 20 and 1 <= it.n_selected_ <= 20
    assert [r["index"] for r in it.importance_ranking_][: it.n_selected_] == it.selected_indices_
    assert it.predict(X[:5]).shape == (5,)
    s = it.summary()
    assert s["n_selected"] == it.n_selected_ and np.isfinite(s["ebm_selected"])
    yb = np.where(X[:, 0] > 0, "yes", "no")
    itb = NoriInterpreter("nori-tiny", regressor_kwargs=dict(weights="random", device="cpu", n_estimators=1),
                          rounds=20, n_repeats=1, reduce_threshold=64).fit(X[:, :6], yb)
    assert itb.task_ == "classification" and not itb.reduced_
    assert set(itb.predict(X[:9, :6])) <= {"yes", "no"}
    p = itb.predict_proba(X[:9, :6])
    np.testing.assert_allclose(p.sum(1), 1.0)


def test_pipeline_cli(tmp_path):
    from synthefy_nori_b200.interpretability.pipeline import main

    rc = main(["--demo", "diabetes", "--model", "nori-tiny", "--weights", "random", "--device", "cpu",
               "--out-dir", str(tmp_path), "--reduce-threshold", "100"])
    assert rc == 0 and (tmp_path / "diabetes.json").exists()


def test_explainability_shim_warns():
    import importlib
    import sys

    sys.modules.pop("synthefy_nori_b200.explainability", None)
    with pytest.warns(DeprecationWarning):
        mod = importlib.import_module("synthefy_nori_b200.explainability")
    assert mod.NoriInterpreter.__name__ == "NoriInterpreter"
