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


def test_analysis_and_model_registry(tmp_path):
    import pandas as pd

    from synthefy_nori_b200.evaluation.analysis import EvalAnalyzer
    from synthefy_nori_b200.evaluation.datasets import DatasetRegistry
    from synthefy_nori_b200.evaluation.models import ModelRegistry, benchmark_list
    from synthefy_nori_b200.evaluation.runner import EvalRunner

    reg = DatasetRegistry(max_train_samples=300)
    reg.load_synthetic(n=300)
    models = ModelRegistry(device="cpu")
    models.add_baselines(["ridge", "knn"])
    models.add_nori("tiny-step100", model="nori-tiny", weights="random", n_estimators=1)
    df = EvalRunner(models.callables(), reg.datasets[:3], str(tmp_path), no_cache=True, verbose=False).run()
    a = EvalAnalyzer(df)
    s = a.summary_by_model()
    assert set(s.index) == {"ridge", "knn", "tiny-step100"}
    h = a.head_to_head("ridge", "knn")
    assert h["wins"] + h["ties"] + h["losses"] == h["n"] == 3
    pw = a.pairwise_comparison()
    assert pw.shape == (3, 3)
    assert list(a.checkpoint_progression("tiny-step")["step"]) == [100]
    assert "Per-model summary" in a.report()
    md = a.markdown_report(str(tmp_path / "r.md"), focus="ridge")
    assert "# Evaluation report" in md
    comp = a.comparison_vs_best_other("ridge")
    assert len(comp) == 3
    assert pd.read_csv(benchmark_list("tabarena_reg"), comment="#", header=None).shape[1] == 2
