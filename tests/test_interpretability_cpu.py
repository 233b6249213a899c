"""Explainers against closed forms on simple predictors, and on a tiny Nori model."""

import numpy as np

from synthefy_nori_b200.interpretability import (ImputationExplainer, distill_glassbox, partial_dependence)
from synthefy_nori_b200.interpretability.glassbox import fit_gam


class _Lin:
    w = np.array([1.0, -2.0, 0.5, 3.0])

    def predict(self, X):
        X = np.asarray(X, np.float64)
        return X @ self.w + 0.7 * X[:, 0] * X[:, 1]


def test_shapley_exact_and_kernel_and_sii():
    m = _Lin()
    bg = np.zeros((10, 4))
    x = np.array([1.0, 2.0, -1.0, 0.5])
    ex = ImputationExplainer(m.predict, bg, index="SV", max_order=1)
    sv = ex.explain(x).values_array(4)
    want = m.w * x + np.array([0.7, 0.7, 0, 0]) * x[0] * x[1] / 2
    np.testing.assert_allclose(sv, want, atol=1e-9)
    lin = lambda X: np.asarray(X, np.float64) @ m.w  # noqa: E731
    kern = ImputationExplainer(lin, bg, random_state=1).explain(x, budget=10).values_array(4)
    np.testing.assert_allclose(kern, m.w * x, atol=1e-6)  # additive model: kernel SHAP is exact
    k2 = ImputationExplainer(m.predict, bg, random_state=1).explain(x, budget=12).values_array(4)
    np.testing.assert_allclose(k2.sum(), m.predict(x[None])[0] - m.predict(bg[:1])[0], atol=1e-6)  # efficiency
    sii = ImputationExplainer(m.predict, bg, index="SII", max_order=2).explain(x)
    np.testing.assert_allclose(sii[(0, 1)], 0.7 * x[0] * x[1], atol=1e-9)
    np.testing.assert_allclose(sii[(2, 3)], 0.0, atol=1e-9)


def test_pdp_linear():
    m = _Lin()
    X = np.random.default_rng(0).standard_normal((50, 4))
    r = partial_dependence(m, X, 3, kind="both", grid_resolution=5)
    g = r["grid_values"][0]
    np.testing.assert_allclose(np.diff(r["average"]) / np.diff(g), 3.0, atol=1e-5)
    assert r["individual"].shape == (50, len(g))
    r2 = partial_dependence(m, X, (0, 1), grid_resolution=4)
    assert r2["average"].shape == (4, 4)


def test_gam_recovers_additive_function():
    rng = np.random.default_rng(0)
    X = rng.uniform(-2, 2, (3000, 3))
    y = np.sin(X[:, 0]) + X[:, 1] ** 2
    gam = fit_gam(X, y, [0, 1, 2], bins=32, rounds=200)
    assert np.corrcoef(gam.predict(X), y)[0, 1] > 0.99
    assert gam.importances(X)[2] < 0.05


def test_distill_tiny_nori():
    from synthefy_nori_b200.api import NoriRegressor

    rng = np.random.default_rng(1)
    X = rng.standard_normal((160, 5)).astype(np.float32)
    y = 2 * X[:, 0] + np.sin(X[:, 1])
    reg = NoriRegressor(model="nori-tiny", weights="random", device="cpu", n_estimators=1).fit(X[:120], y[:120])
    rep = distill_glassbox(reg, X[:120], X[120:], y[120:], n_features=3, rounds=50)
    assert len(rep["features"]) == 3 and np.isfinite(rep["fidelity_r2"])
