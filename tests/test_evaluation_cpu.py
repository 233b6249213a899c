"""Evaluation runner on the offline synthetic suite and a CSV directory."""

import numpy as np
import pandas as pd

from synthefy_nori_b200.evaluation.datasets import DatasetRegistry
from synthefy_nori_b200.evaluation.runner import EvalRunner, compute_reg_metrics


def _ridge(Xtr, ytr, Xte):
    A = np.c_[Xtr, np.ones(len(Xtr))]
    w = np.linalg.lstsq(A.T @ A + 1e-3 * np.eye(A.shape[1]), A.T @ ytr, rcond=None)[0]
    return np.c_[Xte, np.ones(len(Xte))] @ w


def test_runner_synthetic_and_csv(tmp_path):
    d = tmp_path / "data"
    d.mkdir()
    rng = np.random.default_rng(0)
    df = pd.DataFrame({"a": rng.standard_normal(200), "c": rng.choice(["x", "y"], 200)})
    df["target"] = 2 * df["a"] + (df["c"] == "x") + 0.01 * rng.standard_normal(200)
    df.to_csv(d / "toy_train.csv", index=False)
    reg = DatasetRegistry()
    assert reg.load_csv_dir(str(d)) == 1 and reg.load_synthetic(n=300) == 5
    out = tmp_path / "out"
    runner = EvalRunner({"ridge": _ridge}, reg.datasets, str(out))
    res = runner.run()
    assert len(res) == 6 and res["error"].isna().all()
    assert res.set_index("dataset").loc["toy", "r2"] > 0.99
    again = EvalRunner({"ridge": _ridge}, reg.datasets, str(out), verbose=False)
    again.run()
    assert again.cache_hits == 6
    assert (out / "summary.csv").exists()


def test_metrics():
    m = compute_reg_metrics([1, 2, 3], [1, 2, 3])
    assert m["r2"] == 1.0 and m["rmse"] == 0.0
    assert np.isnan(compute_reg_metrics([1], [1])["r2"])
