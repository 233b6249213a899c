"""Local fine-tuning jobs (CPU, tiny model, random base weights): plan, run, report,
checkpoint, deploy behind this build's server and predict through the client."""

import numpy as np
import pandas as pd
import pytest

from synthefy_nori_b200.client.data_models import FineTuneHyperparameters, FineTuneJobRequest, NoriPredictRequest


def _table(tmp_path, n=160):
    rng = np.random.default_rng(0)
    df = pd.DataFrame({"a": rng.standard_normal(n), "b": rng.standard_normal(n),
                       "store": rng.choice(["x", "y"], n)})
    df["target"] = 2 * df["a"] - df["b"] ** 2 + 0.1 * rng.standard_normal(n)
    path = tmp_path / "train.csv"
    df.to_csv(path, index=False)
    return str(path)


def test_hyperparameter_validation():
    with pytest.raises(ValueError):
        FineTuneHyperparameters(model_name="Bad Name!", target_column="t")
    with pytest.raises(ValueError):
        FineTuneHyperparameters(model_name="ok")  # neither target nor tasks
    with pytest.raises(ValueError):
        FineTuneHyperparameters(model_name="ok", target_column="t", time_column="ts")  # needs query_rows
    with pytest.raises(ValueError):
        NoriPredictRequest(X_train=[[1.0]], y_train=[1.0, 2.0], X_test=[[1.0]])


@pytest.mark.timeout(600)
def test_local_fine_tune_deploy_predict(tmp_path):
    from synthefy_nori_b200.finetune import SynthefyNoriFineTuner

    data = _table(tmp_path)
    hp = FineTuneHyperparameters(model_name="ft-test", target_column="target", base_model="nori-tiny",
                                 weights="random", n_steps_per_model=4, validation_every_n_steps=2, batch_size=2,
                                 context_rows=48, query_rows=16, bag=2, lr=1e-3)
    req = FineTuneJobRequest(training_data=data, output_path=str(tmp_path / "out"), hyperparameters=hp)
    with SynthefyNoriFineTuner(device="cpu") as tuner:
        plan = tuner.get_training_plan(req)
        assert plan.n_models == 2 and plan.n_train_rows + plan.n_val_rows == 160 and plan.context_rows == 48
        job = tuner.fine_tune(req)
        job = tuner.wait(job.job_name, timeout_s=500)
        assert job.status == "Completed", job.failure_reason
        rep = tuner.get_training_report(job.job_name)
        assert rep.val_mse_before is not None and rep.val_mse_after is not None and len(rep.curves) == 2
        assert any("validation MSE after" in line for line in tuner.get_logs(job.job_name))
        ep = tuner.deploy(job)
        client = tuner.create_client(ep)
        df = pd.read_csv(data)
        X = df[["a", "b"]].to_numpy(np.float32)
        out = client.predict(X[:100], df["target"].to_numpy()[:100], X[100:110])
        assert np.asarray(out).shape[0] == 10 and np.isfinite(np.asarray(out, float)).all()
        tuner.undeploy(ep)
