"""The SageMaker backend of ``SynthefyNoriFineTuner``: hosted fine-tuning jobs run by the
Nori Algorithm, and asynchronous endpoints that serve their models.

Reference: ``libs/synthefy/src/synthefy/nori_fine_tune.py``, ``_training_jobs.py``,
``_training_artifacts.py``, ``_training_logs.py``, ``_sagemaker_deploy.py``. The flow:

* ``fine_tune``: a local table (file or folder) is uploaded under
  ``<output_path>/<job>/input/``; an ``s3://`` table is used where it is. One
  ``CreateTrainingJob`` runs the Algorithm (``AlgorithmName`` = its ARN) with the job's
  hyperparameters as strings, the ``training`` channel, the output path, the instance type
  and a runtime limit from ``max_training_hours``;
* status / stop / logs: ``DescribeTrainingJob`` (its status names are the job statuses
  here), ``StopTrainingJob``, and the job's CloudWatch streams under
  ``/aws/sagemaker/TrainingJobs`` (``DescribeLogStreams`` + ``GetLogEvents``);
* report and curves: ``training_report.json`` inside the job's ``model.tar.gz``;
* ``deploy``: a model package made from the Algorithm and the job
  (``CreateModelPackage`` with ``SourceAlgorithmSpecification``), a network-isolated model on
  it, an endpoint configuration with ``AsyncInferenceConfig`` (results and failures under
  ``<output_path>/async/``), the endpoint; each step waits for its resource to be ready.
  A failure part way deletes what this call created, newest first, and says so;
* ``undeploy`` deletes the endpoint, its configuration, the model and the package.

Every AWS call goes through client objects with boto3's method names: ``boto3`` builds them
(standard credential chain) unless the caller passes ``sagemaker_client=``, ``s3_client=``
and ``logs_client=`` (the tests pass in-memory fakes).
"""

from __future__ import annotations

import io
import json
import os
import tarfile
import tempfile
import time
import uuid

from synthefy_nori_b200.client.data_models import FineTunedEndpoint, FineTuneJob, FineTuneJobRequest, TrainingReport
from synthefy_nori_b200.client.sagemaker import parse_s3_uri

LOG_GROUP = "/aws/sagemaker/TrainingJobs"
DEFAULT_TRAINING_INSTANCE = "ml.g6e.xlarge"
DEFAULT_INFERENCE_INSTANCE = "ml.g6e.xlarge"
TERMINAL = ("Completed", "Failed", "Stopped")


class SageMakerFineTuningError(RuntimeError):
    pass


def _hyperparameters(hp) -> dict:
    """The Algorithm takes string-valued hyperparameters; nested values travel as JSON."""
    out = {}
    for k, v in hp.model_dump(exclude_none=True).items():
        out[k] = v if isinstance(v, str) else json.dumps(v)
    return out


class SageMakerJobs:
    def __init__(self, *, region_name=None, sagemaker_client=None, s3_client=None, logs_client=None,
                 poll_s: float = 15.0):
        if sagemaker_client is None or s3_client is None or logs_client is None:
            try:
                import boto3
            except ImportError as exc:
                raise ImportError("the sagemaker backend needs boto3 and AWS credentials (or sagemaker_client=, "
                                  "s3_client= and logs_client=); use backend='local' to fine-tune on this "
                                  "machine's GPUs") from exc
            session = boto3.Session(region_name=region_name)
            sagemaker_client = sagemaker_client or session.client("sagemaker")
            s3_client = s3_client or session.client("s3")
            logs_client = logs_client or session.client("logs")
        self.sm, self.s3, self.logs = sagemaker_client, s3_client, logs_client
        self.poll_s = float(poll_s)
        self._requests: dict[str, FineTuneJobRequest] = {}
        self._endpoints: dict[str, dict] = {}

    # ---------------------------------------------------------------- jobs
    def _stage_input(self, request: FineTuneJobRequest, job_name: str) -> str:
        src = request.training_data
        if src.startswith("s3://"):
            return src
        if not os.path.exists(src):
            raise SageMakerFineTuningError(f"training data {src!r} does not exist")
        bucket, prefix = parse_s3_uri(request.output_path)
        base = "/".join(p for p in (prefix.strip("/"), job_name, "input") if p)
        files = [src] if os.path.isfile(src) else sorted(
            os.path.join(d, f) for d, _, fs in os.walk(src) for f in fs if f.endswith((".csv", ".parquet", ".pq")))
        if not files:
            raise SageMakerFineTuningError(f"no CSV or Parquet files under {src!r}")
        root = src if os.path.isdir(src) else os.path.dirname(src)
        for f in files:
            self.s3.upload_file(f, bucket, f"{base}/{os.path.relpath(f, root)}")
        return f"s3://{bucket}/{base}/"

    def fine_tune(self, request: FineTuneJobRequest) -> FineTuneJob:
        if not request.algorithm or not request.role_arn:
            raise SageMakerFineTuningError("the sagemaker backend needs algorithm= (the Nori Algorithm ARN) and "
                                           "role_arn= (an execution role SageMaker can assume)")
        parse_s3_uri(request.output_path)
        hp = request.hyperparameters
        job_name = request.job_name or f"nori-ft-{hp.model_name}-{uuid.uuid4().hex[:8]}"[:63]
        data = self._stage_input(request, job_name)
        limit = int(3600 * (hp.max_training_hours or 24.0))
        self.sm.create_training_job(
            TrainingJobName=job_name,
            AlgorithmSpecification={"AlgorithmName": request.algorithm, "TrainingInputMode": "File"},
            RoleArn=request.role_arn,
            HyperParameters=_hyperparameters(hp),
            InputDataConfig=[{"ChannelName": "training", "DataSource": {"S3DataSource": {
                "S3DataType": "S3Prefix", "S3Uri": data, "S3DataDistributionType": "FullyReplicated"}}}],
            OutputDataConfig={"S3OutputPath": request.output_path.rstrip("/") + "/"},
            ResourceConfig={"InstanceType": request.instance_type or DEFAULT_TRAINING_INSTANCE, "InstanceCount": 1,
                            "VolumeSizeInGB": 100},
            StoppingCondition={"MaxRuntimeInSeconds": limit},
        )
        self._requests[job_name] = request
        return FineTuneJob(job_name=job_name, status="InProgress", backend="sagemaker", created_at=time.time(),
                           model_name=hp.model_name)

    def get_status(self, job_name: str) -> FineTuneJob:
        d = self.sm.describe_training_job(TrainingJobName=job_name)
        status = d.get("TrainingJobStatus", "InProgress")
        if status not in ("InProgress", "Completed", "Failed", "Stopping", "Stopped"):
            status = "InProgress"
        hp = d.get("HyperParameters") or {}
        created, ended = d.get("CreationTime"), d.get("TrainingEndTime")
        stamp = (lambda t: t.timestamp() if hasattr(t, "timestamp") else float(t) if t is not None else None)
        return FineTuneJob(job_name=job_name, status=status, backend="sagemaker",
                           created_at=stamp(created) or time.time(), ended_at=stamp(ended),
                           model_artifact=(d.get("ModelArtifacts") or {}).get("S3ModelArtifacts"),
                           failure_reason=d.get("FailureReason"), model_name=hp.get("model_name", job_name))

    def wait(self, job_name: str, *, poll_s: float | None = None, timeout_s: float | None = None) -> FineTuneJob:
        t0 = time.monotonic()
        while True:
            job = self.get_status(job_name)
            if job.status in TERMINAL:
                return job
            if timeout_s is not None and time.monotonic() - t0 > timeout_s:
                raise TimeoutError(f"job {job_name} still {job.status} after {timeout_s} s")
            time.sleep(self.poll_s if poll_s is None else poll_s)

    def stop(self, job_name: str) -> FineTuneJob:
        self.sm.stop_training_job(TrainingJobName=job_name)
        return self.get_status(job_name)

    def get_logs(self, job_name: str, *, follow: bool = False, poll_s: float | None = None):
        """The job's CloudWatch log lines, oldest first, across its streams; with ``follow``
        keeps reading until the job ends."""
        tokens: dict[str, str | None] = {}
        while True:
            streams = self.logs.describe_log_streams(logGroupName=LOG_GROUP, logStreamNamePrefix=job_name + "/")
            for s in streams.get("logStreams", []):
                name = s["logStreamName"]
                while True:
                    kw = dict(logGroupName=LOG_GROUP, logStreamName=name, startFromHead=True)
                    if tokens.get(name):
                        kw["nextToken"] = tokens[name]
                    r = self.logs.get_log_events(**kw)
                    for e in r.get("events", []):
                        yield e.get("message", "")
                    nxt = r.get("nextForwardToken")
                    if nxt is None or nxt == tokens.get(name):
                        tokens[name] = nxt
                        break
                    tokens[name] = nxt
            if not follow or self.get_status(job_name).status in TERMINAL:
                return
            time.sleep(self.poll_s if poll_s is None else poll_s)

    def get_training_report(self, job_name: str) -> TrainingReport:
        job = self.get_status(job_name)
        if job.status != "Completed" or not job.model_artifact:
            raise SageMakerFineTuningError(f"job {job_name} has no model artifact yet (status {job.status})")
        bucket, key = parse_s3_uri(job.model_artifact)
        fd, path = tempfile.mkstemp(suffix=".tar.gz")
        os.close(fd)
        try:
            self.s3.download_file(bucket, key, path)
            with tarfile.open(path, "r:gz") as tar:
                member = next((m for m in tar.getmembers()
                               if os.path.basename(m.name) == "training_report.json" and m.isfile()), None)
                if member is None:
                    raise SageMakerFineTuningError(f"{job.model_artifact} holds no training_report.json")
                raw = tar.extractfile(member).read()
        finally:
            os.unlink(path)
        return TrainingReport.model_validate(json.load(io.BytesIO(raw)))

    # ---------------------------------------------------------------- endpoints
    def _wait_for(self, describe, key: str, ready: str, failed: tuple, what: str, timeout_s: float):
        t0 = time.monotonic()
        while True:
            d = describe()
            status = d.get(key)
            if status == ready:
                return d
            if status in failed:
                raise SageMakerFineTuningError(f"{what} ended {status}: {d.get('FailureReason', 'no reason given')}")
            if time.monotonic() - t0 > timeout_s:
                raise TimeoutError(f"{what} not {ready} after {timeout_s} s (status {status})")
            time.sleep(self.poll_s)

    def deploy(self, job_name: str, *, endpoint_name: str | None = None, instance_type: str | None = None,
               algorithm: str | None = None, role_arn: str | None = None, output_path: str | None = None,
               timeout_s: float = 3600.0) -> FineTunedEndpoint:
        job = self.get_status(job_name)
        if job.status != "Completed" or not job.model_artifact:
            raise SageMakerFineTuningError(f"job {job_name} has no completed model to deploy (status {job.status})")
        req = self._requests.get(job_name)
        algorithm = algorithm or (req.algorithm if req else None)
        role_arn = role_arn or (req.role_arn if req else None)
        output_path = (output_path or (req.output_path if req else "")).rstrip("/")
        if not algorithm or not role_arn or not output_path:
            raise SageMakerFineTuningError("deploy needs the job's algorithm=, role_arn= and output_path=")
        name = (endpoint_name or f"{job.model_name}-ep")[:63]
        created: list[tuple[str, str]] = []
        try:
            pkg = self.sm.create_model_package(
                ModelPackageName=name, ModelPackageDescription=f"Nori fine-tuned by {job_name}",
                SourceAlgorithmSpecification={"SourceAlgorithms": [
                    {"AlgorithmName": algorithm, "ModelDataUrl": job.model_artifact}]},
                CertifyForMarketplace=False)["ModelPackageArn"]
            created.append(("model_package", pkg))
            self._wait_for(lambda: self.sm.describe_model_package(ModelPackageName=pkg), "ModelPackageStatus",
                           "Completed", ("Failed", "Deleting"), f"model package {pkg}", timeout_s)
            self.sm.create_model(ModelName=name, PrimaryContainer={"ModelPackageName": pkg},
                                 ExecutionRoleArn=role_arn, EnableNetworkIsolation=True)
            created.append(("model", name))
            self.sm.create_endpoint_config(
                EndpointConfigName=name,
                ProductionVariants=[{"VariantName": "AllTraffic", "ModelName": name, "InitialInstanceCount": 1,
                                     "InstanceType": instance_type or DEFAULT_INFERENCE_INSTANCE}],
                AsyncInferenceConfig={"OutputConfig": {"S3OutputPath": f"{output_path}/async/output",
                                                       "S3FailurePath": f"{output_path}/async/failure"}})
            created.append(("endpoint_config", name))
            self.sm.create_endpoint(EndpointName=name, EndpointConfigName=name)
            created.append(("endpoint", name))
            self._wait_for(lambda: self.sm.describe_endpoint(EndpointName=name), "EndpointStatus", "InService",
                           ("Failed", "OutOfService", "Deleting"), f"endpoint {name}", timeout_s)
        except Exception as exc:
            left = self._delete(created)
            note = "" if not left else f"; could not delete: {', '.join(left)}"
            raise SageMakerFineTuningError(f"deploy of {job_name} failed ({exc}); removed what it created{note}") from exc
        self._endpoints[name] = {"created": created, "staging": f"{output_path}/async/requests"}
        return FineTunedEndpoint(endpoint_name=name, url=f"sagemaker://{name}", model_name=job.model_name,
                                 model_artifact=job.model_artifact, backend="sagemaker")

    def _delete(self, created) -> list[str]:
        calls = {"endpoint": lambda v: self.sm.delete_endpoint(EndpointName=v),
                 "endpoint_config": lambda v: self.sm.delete_endpoint_config(EndpointConfigName=v),
                 "model": lambda v: self.sm.delete_model(ModelName=v),
                 "model_package": lambda v: self.sm.delete_model_package(ModelPackageName=v)}
        left = []
        for kind, value in reversed(created):
            try:
                calls[kind](value)
            except Exception:  # noqa: BLE001 - reported to the caller by name
                left.append(f"{kind} {value}")
        return left

    def undeploy(self, endpoint_name: str) -> None:
        rec = self._endpoints.pop(endpoint_name, None)
        created = rec["created"] if rec else [("endpoint_config", endpoint_name), ("endpoint", endpoint_name)]
        left = self._delete(created)
        if left:
            raise SageMakerFineTuningError(f"could not delete: {', '.join(left)}")

    def staging_uri(self, endpoint_name: str) -> str | None:
        rec = self._endpoints.get(endpoint_name)
        return rec["staging"] if rec else None
