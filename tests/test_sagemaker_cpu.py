"""SageMaker mode of the client against in-memory fakes of S3 and the SageMaker runtime
whose endpoint is this framework's own container app (``POST /invocations`` with the
request tensor file), on CPU."""

import os

import numpy as np
import pytest


class _ClientError(Exception):
    """Shaped like botocore's ClientError for a missing object."""

    def __init__(self, code="404"):
        super().__init__(code)
        self.response = {"Error": {"Code": code}, "ResponseMetadata": {"HTTPStatusCode": 404}}


class FakeS3:
    def __init__(self):
        self.objects: dict = {}
        self.deleted: list = []

    def upload_file(self, path, bucket, key):
        with open(path, "rb") as f:
            self.objects[(bucket, key)] = f.read()

    def head_object(self, Bucket, Key):
        if (Bucket, Key) not in self.objects:
            raise _ClientError()
        return {"ContentLength": len(self.objects[(Bucket, Key)])}

    def download_file(self, bucket, key, path):
        with open(path, "wb") as f:
            f.write(self.objects[(bucket, key)])

    def delete_object(self, Bucket, Key):
        self.deleted.append(f"s3://{Bucket}/{Key}")
        self.objects.pop((Bucket, Key), None)


class FakeRuntime:
    """Asynchronous endpoint: reads the input object, runs the container app, writes
    result.json (or a failure object) under the invocation's output prefix."""

    def __init__(self, s3, app, *, out="s3://out-bucket/async", fail=False, never=False):
        from starlette.testclient import TestClient

        self.s3, self.http, self.out, self.fail, self.never = s3, TestClient(app), out, fail, never
        self.calls = []

    def invoke_endpoint_async(self, **kw):
        from synthefy_nori_b200.client.sagemaker import parse_s3_uri

        self.calls.append(kw)
        inv = kw["InferenceId"]
        output = f"{self.out}/{kw['S3OutputPathExtension']}/{kw['Filename']}"
        failure = f"{self.out}/{kw['S3OutputPathExtension']}/failure.json"
        if not self.never:
            body = self.s3.objects[parse_s3_uri(kw["InputLocation"])]
            if self.fail:
                self.s3.objects[parse_s3_uri(failure)] = b'{"ErrorMessage": "model server crashed"}'
            else:
                r = self.http.post("/invocations", content=body, headers={"content-type": kw["ContentType"]})
                assert r.status_code == 200, r.text
                self.s3.objects[parse_s3_uri(output)] = r.content
        return {"InferenceId": inv, "OutputLocation": output, "FailureLocation": failure}


@pytest.fixture(scope="module")
def app():
    from synthefy_nori_b200.serving import create_app

    return create_app(default_model="nori-tiny", weights="random", device="cpu")


def _data():
    rng = np.random.default_rng(0)
    X = rng.standard_normal((70, 4)).astype(np.float32)
    X[3, 1] = np.nan
    y = X[:, 0] * 2 + 0.1 * rng.standard_normal(70)
    return X[:50], y[:50], X[50:]


def test_tensorfile_round_trip(tmp_path):
    from synthefy_nori_b200.client.sagemaker import HEADER_BYTES, read_tensorfile, write_tensorfile

    Xtr, ytr, Xte = _data()
    p = tmp_path / "r.tensorfile"
    n = write_tensorfile(p, {"X_train": Xtr, "y_train": ytr, "X_test": Xte}, {"model": "nori-tiny", "quantiles": [0.1]})
    assert os.path.getsize(p) == n == HEADER_BYTES + Xtr.nbytes + ytr.astype(np.float64).nbytes + Xte.nbytes
    raw = p.read_bytes()
    assert raw[:8] == b"NORI_REQ"
    arrays, meta = read_tensorfile(p)
    np.testing.assert_array_equal(arrays["X_train"], Xtr)  # NaN positions included
    np.testing.assert_array_equal(arrays["y_train"], ytr)
    assert meta == {"model": "nori-tiny", "quantiles": [0.1]}
    bad = tmp_path / "bad.tensorfile"
    bad.write_bytes(b"NOT_NORI" + raw[8:])
    with pytest.raises(ValueError):
        read_tensorfile(bad)


def test_sagemaker_mode_matches_local(app):
    from synthefy_nori_b200.client import SynthefyNoriClient

    Xtr, ytr, Xte = _data()
    s3 = FakeS3()
    rt = FakeRuntime(s3, app)
    local = SynthefyNoriClient(mode="local", model="nori-tiny", weights="random", device="cpu")
    sm = SynthefyNoriClient(mode="sagemaker", model="nori-tiny", endpoint_name="nori-ep",
                            s3_staging_uri="s3://stage-bucket/nori/requests", sagemaker_runtime_client=rt,
                            s3_client=s3)
    np.testing.assert_allclose(sm.predict(Xtr, ytr, Xte), local.predict(Xtr, ytr, Xte), rtol=1e-5, atol=1e-5)
    q = sm.predict(Xtr, ytr, Xte, output_type="quantiles", quantiles=[0.1, 0.9])
    assert q.shape == (2, 20)
    call = rt.calls[0]
    assert call["EndpointName"] == "nori-ep" and call["ContentType"] == "application/vnd.synthefy.nori.tensorfile"
    assert call["InputLocation"].startswith(f"s3://stage-bucket/nori/requests/nori-ep/{call['InferenceId']}/")
    # every staged object of a finished call is deleted
    assert not s3.objects
    assert any(d.endswith("request.tensorfile") for d in s3.deleted)
    with pytest.raises(ValueError):
        sm.predict(Xtr, np.r_[ytr[:-1], np.nan], Xte)


def test_sagemaker_failure_and_timeout(app):
    from synthefy_nori_b200.client import APITimeoutError, SageMakerInvocationError, SynthefyNoriClient

    Xtr, ytr, Xte = _data()
    s3 = FakeS3()
    bad = SynthefyNoriClient(mode="sagemaker", model="nori-tiny", endpoint_name="ep", s3_staging_uri="s3://b/p",
                             sagemaker_runtime_client=FakeRuntime(s3, app, fail=True), s3_client=s3)
    with pytest.raises(SageMakerInvocationError, match="model server crashed"):
        bad.predict(Xtr, ytr, Xte)
    s3b = FakeS3()
    slow = SynthefyNoriClient(mode="sagemaker", model="nori-tiny", endpoint_name="ep", s3_staging_uri="s3://b/p",
                              sagemaker_runtime_client=FakeRuntime(s3b, app, never=True), s3_client=s3b, timeout=0.3)
    slow.sagemaker.poll_initial = 0.05
    with pytest.raises(APITimeoutError):
        slow.predict(Xtr, ytr, Xte)
    # the outcome is unknown: the staged input stays for the bucket's lifecycle rule
    assert any(k[1].endswith("request.tensorfile") for k in s3b.objects)


def test_sagemaker_refuses_foreign_output_prefix(app):
    from synthefy_nori_b200.client import SynthefyNoriClient

    Xtr, ytr, Xte = _data()
    s3 = FakeS3()
    rt = FakeRuntime(s3, app)
    orig = rt.invoke_endpoint_async

    def elsewhere(**kw):
        r = orig(**kw)
        r["OutputLocation"] = "s3://out-bucket/async/someone-else/result.json"
        return r

    rt.invoke_endpoint_async = elsewhere
    c = SynthefyNoriClient(mode="sagemaker", model="nori-tiny", endpoint_name="ep", s3_staging_uri="s3://b/p",
                           sagemaker_runtime_client=rt, s3_client=s3)
    with pytest.raises(RuntimeError, match="outside this invocation"):
        c.predict(Xtr, ytr, Xte)


def test_container_routes_accept_json_and_tensorfile(app, tmp_path):
    from starlette.testclient import TestClient

    from synthefy_nori_b200.client.sagemaker import CONTENT_TYPE, write_tensorfile

    http = TestClient(app)
    assert http.get("/ping").status_code == 200
    Xtr, ytr, Xte = _data()
    p = tmp_path / "r.tensorfile"
    write_tensorfile(p, {"X_train": Xtr, "y_train": ytr, "X_test": Xte}, {"model": "nori-tiny"})
    r1 = http.post("/invocations", content=p.read_bytes(), headers={"content-type": CONTENT_TYPE})
    rows = [[None if not np.isfinite(v) else float(v) for v in r] for r in Xtr]
    body = {"X_train": rows, "y_train": ytr.tolist(), "X_test": Xte.tolist(), "model": "nori-tiny"}
    r2 = http.post("/invocations", json=body)
    assert r1.status_code == r2.status_code == 200
    np.testing.assert_allclose(r1.json()["predictions"], r2.json()["predictions"], rtol=1e-5, atol=1e-5)
    # bad metadata is a 422, not a crash
    write_tensorfile(p, {"X_train": Xtr, "y_train": ytr, "X_test": Xte}, {"model": "nori-tiny", "task": "cls"})
    assert http.post("/invocations", content=p.read_bytes(), headers={"content-type": CONTENT_TYPE}).status_code == 422


class FakeSageMaker:
    """Control plane: a training job that completes on the second describe, with a model
    artifact holding training_report.json; packages, models, configs and endpoints."""

    def __init__(self, s3, *, endpoint_fails=False):
        self.s3, self.endpoint_fails = s3, endpoint_fails
        self.jobs, self.resources, self.calls = {}, {}, []

    def create_training_job(self, **kw):
        self.calls.append(("create_training_job", kw))
        self.jobs[kw["TrainingJobName"]] = {"kw": kw, "describes": 0, "stopped": False}

    def describe_training_job(self, TrainingJobName):
        import io
        import json
        import tarfile

        j = self.jobs[TrainingJobName]
        j["describes"] += 1
        base = {"TrainingJobName": TrainingJobName, "HyperParameters": j["kw"]["HyperParameters"], "CreationTime": 1.0}
        if j["stopped"]:
            return {**base, "TrainingJobStatus": "Stopped"}
        if j["describes"] < 2:
            return {**base, "TrainingJobStatus": "InProgress"}
        out = j["kw"]["OutputDataConfig"]["S3OutputPath"] + f"{TrainingJobName}/output/model.tar.gz"
        bucket, key = out[5:].split("/", 1)
        if (bucket, key) not in self.s3.objects:
            buf = io.BytesIO()
            with tarfile.open(fileobj=buf, mode="w:gz") as tar:
                raw = json.dumps({"val_mse_before": 2.0, "val_mse_after": 1.0, "best_step": [7]}).encode()
                info = tarfile.TarInfo("training_report.json")
                info.size = len(raw)
                tar.addfile(info, io.BytesIO(raw))
            self.s3.objects[(bucket, key)] = buf.getvalue()
        return {**base, "TrainingJobStatus": "Completed", "TrainingEndTime": 2.0,
                "ModelArtifacts": {"S3ModelArtifacts": out}}

    def stop_training_job(self, TrainingJobName):
        self.jobs[TrainingJobName]["stopped"] = True

    def create_model_package(self, **kw):
        arn = f"arn:aws:sagemaker:us-east-1:1:model-package/{kw['ModelPackageName']}"
        self.resources[("model_package", arn)] = kw
        return {"ModelPackageArn": arn}

    def describe_model_package(self, ModelPackageName):
        return {"ModelPackageStatus": "Completed"}

    def create_model(self, **kw):
        self.resources[("model", kw["ModelName"])] = kw

    def create_endpoint_config(self, **kw):
        self.resources[("endpoint_config", kw["EndpointConfigName"])] = kw

    def create_endpoint(self, **kw):
        self.resources[("endpoint", kw["EndpointName"])] = kw

    def describe_endpoint(self, EndpointName):
        return {"EndpointStatus": "Failed" if self.endpoint_fails else "InService", "FailureReason": "capacity"}

    def delete_endpoint(self, EndpointName):
        del self.resources[("endpoint", EndpointName)]

    def delete_endpoint_config(self, EndpointConfigName):
        del self.resources[("endpoint_config", EndpointConfigName)]

    def delete_model(self, ModelName):
        del self.resources[("model", ModelName)]

    def delete_model_package(self, ModelPackageName):
        del self.resources[("model_package", ModelPackageName)]


class FakeLogs:
    def describe_log_streams(self, logGroupName, logStreamNamePrefix):
        assert logGroupName == "/aws/sagemaker/TrainingJobs"
        return {"logStreams": [{"logStreamName": logStreamNamePrefix + "algo-1"}]}

    def get_log_events(self, logGroupName, logStreamName, startFromHead, nextToken=None):
        if nextToken is None:
            return {"events": [{"message": "step 1 loss 0.5"}, {"message": "step 2 loss 0.4"}], "nextForwardToken": "t1"}
        return {"events": [], "nextForwardToken": "t1"}


def test_sagemaker_fine_tuning_job_deploy_and_predict(app, tmp_path):
    import pandas as pd

    from synthefy_nori_b200.client.data_models import FineTuneHyperparameters, FineTuneJobRequest
    from synthefy_nori_b200.finetune import SynthefyNoriFineTuner

    Xtr, ytr, Xte = _data()
    table = tmp_path / "data"
    table.mkdir()
    pd.DataFrame({"a": Xtr[:, 0], "b": Xtr[:, 2], "y": ytr}).to_csv(table / "t.csv", index=False)
    s3 = FakeS3()
    sm = FakeSageMaker(s3)
    tuner = SynthefyNoriFineTuner(backend="sagemaker", sagemaker_client=sm, s3_client=s3, logs_client=FakeLogs(),
                                  poll_s=0.0)
    req = FineTuneJobRequest(training_data=str(table), output_path="s3://ft-bucket/runs",
                             hyperparameters=FineTuneHyperparameters(target_column="y", model_name="nori-tiny",
                                                                     base_model="nori-tiny", max_training_hours=2.0),
                             backend="sagemaker", algorithm="arn:aws:sagemaker:us-east-1:1:algorithm/nori",
                             role_arn="arn:aws:iam::1:role/sm", job_name="job-1")
    job = tuner.fine_tune(req)
    assert job.status == "InProgress" and job.backend == "sagemaker"
    kw = sm.calls[0][1]
    assert kw["AlgorithmSpecification"]["AlgorithmName"].endswith("algorithm/nori")
    assert kw["StoppingCondition"]["MaxRuntimeInSeconds"] == 7200
    assert kw["HyperParameters"]["target_column"] == "y" and isinstance(kw["HyperParameters"]["bag"], str)
    assert ("ft-bucket", "runs/job-1/input/t.csv") in s3.objects  # the local table was staged
    done = tuner.wait("job-1", poll_s=0.0, timeout_s=5)
    assert done.status == "Completed" and done.model_artifact.endswith("model.tar.gz")
    assert list(tuner.get_logs("job-1")) == ["step 1 loss 0.5", "step 2 loss 0.4"]
    rep = tuner.get_training_report("job-1")
    assert rep.val_mse_after == 1.0 and rep.best_step == [7]
    ep = tuner.deploy("job-1", endpoint_name="nori-ft-ep")
    assert ep.backend == "sagemaker" and ("endpoint", "nori-ft-ep") in sm.resources
    cfg = sm.resources[("endpoint_config", "nori-ft-ep")]
    assert cfg["AsyncInferenceConfig"]["OutputConfig"]["S3OutputPath"] == "s3://ft-bucket/runs/async/output"
    client = tuner.create_client(ep, sagemaker_runtime_client=FakeRuntime(s3, app))
    pred = client.predict(Xtr, ytr, Xte)
    assert pred.shape == (20,) and np.all(np.isfinite(pred))
    tuner.undeploy(ep)
    assert not sm.resources


def test_sagemaker_deploy_failure_removes_what_it_made():
    from synthefy_nori_b200.finetune.sagemaker import SageMakerFineTuningError, SageMakerJobs

    s3 = FakeS3()
    sm = FakeSageMaker(s3, endpoint_fails=True)
    jobs = SageMakerJobs(sagemaker_client=sm, s3_client=s3, logs_client=FakeLogs(), poll_s=0.0)
    sm.jobs["j"] = {"kw": {"HyperParameters": {"model_name": "m"}, "OutputDataConfig": {"S3OutputPath": "s3://b/o/"}},
                    "describes": 5, "stopped": False}
    with pytest.raises(SageMakerFineTuningError, match="capacity"):
        jobs.deploy("j", algorithm="arn:alg", role_arn="arn:role", output_path="s3://b/o")
    assert not sm.resources
