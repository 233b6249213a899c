"""Wire and job data models of the client SDK (pydantic).

The request / response models are the hosted API's JSON contract (the same field names
as the reference's ``libs/synthefy/src/synthefy/data_models.py`` and
``nori_data_models.py``, so payloads written for either work against both); the
server (``synthefy_nori_b200.serving``) validates requests with them and the client
builds them.  The memory / large-context report models describe what ``predict`` did.
The fine-tuning models describe a job of ``SynthefyNoriFineTuner`` (``finetune``).
"""

from __future__ import annotations

import re
from typing import Literal, Optional, Union

from pydantic import BaseModel, ConfigDict, Field, field_validator, model_validator

OUTPUT_TYPES = ("mean", "median", "mode", "quantiles", "full")
MODEL_NAME_RULE = re.compile(r"^[a-z0-9][a-z0-9-]{0,62}$")


class MemoryAttempt(BaseModel):
    rung: str
    outcome: Literal["success", "oom", "skipped"]
    detail: Optional[str] = None


class MemoryReport(BaseModel):
    """The cache rung ``predict`` ended on and how it got there."""

    rung: Optional[str] = None
    cache_dtype: Optional[str] = None
    est_cache_gb: Optional[float] = None
    resident_gb: Optional[float] = None
    dropped_context_rows: int = 0
    query_chunk: Optional[int] = None
    attempts: list[MemoryAttempt] = Field(default_factory=list)

    @classmethod
    def from_policy(cls, pol) -> "MemoryReport":
        if pol is None:
            return cls()
        dtype = pol.placement()[0] if pol.rung else pol.cache_dtype
        return cls(rung=pol.rung, cache_dtype=dtype, est_cache_gb=pol.est_cache_gb, resident_gb=pol.resident_gb,
                   dropped_context_rows=pol.dropped_context_rows, query_chunk=pol.query_chunk,
                   attempts=[MemoryAttempt(rung=pol.rung or "none", outcome="success")])


class MultiTargetMemoryReport(MemoryReport):
    target_index: int = 0


class LargeContextReport(BaseModel):
    policy: Optional[str] = None
    threshold: Optional[int] = None
    n_context_rows: Optional[int] = None
    n_used_rows: Optional[int] = None
    detail: Optional[dict] = None


class MultiTargetPredictionPolicy(BaseModel):
    model_config = ConfigDict(extra="forbid")
    strategy: Literal["independent", "copula", "autoregressive"] = "independent"
    n_samples: int = Field(256, ge=1, le=100_000)
    seed: int = Field(0, ge=0)


class NoriPredictOptions(BaseModel):
    """Everything of a prediction request except its arrays (the metadata of a request
    tensor file carries exactly these fields)."""

    model_config = ConfigDict(extra="forbid")
    task: str = "regression"
    model: Optional[str] = None
    output_type: Optional[str] = None
    quantiles: Optional[list[float]] = None
    discretize: Optional[str] = None
    categorical_levels: Optional[list[float]] = None
    memory_policy: Optional[Union[str, dict]] = None
    large_context_policy: Optional[Union[str, list[str]]] = None
    large_context_threshold: Optional[int] = Field(None, ge=1)
    large_context_seed: Optional[int] = Field(None, ge=0)
    multi_target_prediction_strategy: Optional[str] = None
    multi_target_prediction_policy: Optional[dict] = None

    @field_validator("task")
    @classmethod
    def _task(cls, v):
        if v != "regression":
            raise ValueError("only task='regression' is supported")
        return v

    @field_validator("output_type")
    @classmethod
    def _out(cls, v):
        if v is not None and v not in OUTPUT_TYPES:
            raise ValueError(f"output_type must be one of {OUTPUT_TYPES}")
        return v

    @field_validator("quantiles")
    @classmethod
    def _q(cls, v):
        if v is not None and any(not 0.0 < q < 1.0 for q in v):
            raise ValueError("quantiles must lie in (0, 1)")
        return v


class NoriPredictRequest(NoriPredictOptions):
    """One prediction request: context ``X_train`` / ``y_train``, query ``X_test``."""

    X_train: list[list[Optional[float]]]
    y_train: Union[list[float], list[list[float]]]
    X_test: list[list[Optional[float]]]

    @model_validator(mode="after")
    def _shapes(self):
        n, f = len(self.X_train), len(self.X_train[0]) if self.X_train else 0
        if n == 0 or len(self.X_test) == 0:
            raise ValueError("X_train and X_test need at least one row")
        if len(self.y_train) != n:
            raise ValueError("y_train must have one entry per X_train row")
        if any(len(r) != f for r in self.X_train) or any(len(r) != f for r in self.X_test):
            raise ValueError("every row of X_train and X_test needs the same number of features")
        return self


class NoriPredictResponse(BaseModel):
    task: str = "regression"
    predictions: Union[list[Optional[float]], list[list[Optional[float]]]]
    model: Optional[str] = None
    model_version: Optional[str] = None
    memory_report: Optional[MemoryReport] = None
    multi_target_memory_reports: Optional[list[MultiTargetMemoryReport]] = None
    discretize: Optional[str] = None
    output_type: Optional[str] = None
    quantiles: Optional[list[list[Optional[float]]]] = None
    taus: Optional[list[float]] = None
    large_context_report: Optional[LargeContextReport] = None
    samples: Optional[list[list[list[Optional[float]]]]] = None
    multi_target_prediction_strategy: Optional[str] = None
    target_orders: Optional[list[list[int]]] = None


# ------------------------------------------------------------------ fine-tuning
class TaskTable(BaseModel):
    model_config = ConfigDict(extra="forbid")
    path: str
    target_column: str
    feature_columns: Optional[list[str]] = None
    task_column: Optional[str] = None
    time_column: Optional[str] = None


class FineTuneHyperparameters(BaseModel):
    """What a fine-tuning job trains: target / features of the table(s), the base model,
    episode sizes, bagging, learning rate, early stopping and budget."""

    model_config = ConfigDict(extra="forbid", protected_namespaces=())
    target_column: Optional[str] = Field(None, min_length=1)
    model_name: str
    base_model: str = "nori-6m"
    task: Literal["regression"] = "regression"
    feature_columns: Optional[list[str]] = None
    task_column: Optional[str] = None
    time_column: Optional[str] = None
    context_rows: Optional[Union[int, dict[str, float]]] = None
    query_rows: Optional[Union[int, dict[str, float]]] = None
    tasks: Optional[list[TaskTable]] = None
    bag: int = Field(1, ge=1, le=64, description="models trained on different row partitions, averaged at predict")
    n_steps_per_model: int = Field(200, ge=1)
    batch_size: int = Field(8, ge=1, description="episodes per optimizer step")
    lr: float = Field(1e-5, gt=0)
    patience: Optional[int] = Field(None, ge=1, description="validations without improvement before stopping")
    validation_every_n_steps: int = Field(25, ge=1)
    validation_fraction: float = Field(0.2, gt=0, lt=1)
    max_training_hours: Optional[float] = Field(None, gt=0)
    weights: Optional[str] = Field(None, description="'random' to start from random weights (offline tests)")
    seed: int = Field(0, ge=0)

    @field_validator("model_name")
    @classmethod
    def _name(cls, v):
        if not MODEL_NAME_RULE.match(v):
            raise ValueError("model_name: lowercase letters, digits and '-', starting with a letter or digit, <= 63")
        return v

    @model_validator(mode="after")
    def _target(self):
        if (self.target_column is None) == (self.tasks is None):
            raise ValueError("set exactly one of target_column and tasks")
        if self.time_column is not None and self.query_rows is None:
            raise ValueError("time_column needs query_rows")
        return self


class FineTuneJobRequest(BaseModel):
    model_config = ConfigDict(extra="forbid")
    training_data: str = Field(description="a CSV / Parquet file or a folder of them (local path or s3:// URI)")
    output_path: str
    hyperparameters: FineTuneHyperparameters
    backend: Literal["local", "sagemaker"] = "local"
    algorithm: Optional[str] = Field(None, description="SageMaker Algorithm ARN (sagemaker backend)")
    role_arn: Optional[str] = None
    instance_type: Optional[str] = None
    job_name: Optional[str] = None


class ChildCurve(BaseModel):
    model_index: int
    steps: list[int] = Field(default_factory=list)
    train_loss: list[float] = Field(default_factory=list)
    val_mse: list[float] = Field(default_factory=list)


class TrainingPlan(BaseModel):
    n_models: int
    n_train_rows: int
    n_val_rows: int
    n_features: int
    steps_per_model: int
    context_rows: int
    query_rows: int


class TaskScore(BaseModel):
    task: str
    val_mse_before: float
    val_mse_after: float


class TrainingReport(BaseModel):
    val_mse_before: Optional[float] = None
    val_mse_after: Optional[float] = None
    best_step: list[int] = Field(default_factory=list)
    curves: list[ChildCurve] = Field(default_factory=list)
    task_scores: list[TaskScore] = Field(default_factory=list)
    stopped_early: bool = False


class FineTuneJob(BaseModel):
    job_name: str
    status: Literal["Pending", "InProgress", "Completed", "Failed", "Stopping", "Stopped"]
    backend: str = "local"
    created_at: float
    ended_at: Optional[float] = None
    model_artifact: Optional[str] = None
    failure_reason: Optional[str] = None
    model_name: str


class FineTunedEndpoint(BaseModel):
    endpoint_name: str
    url: str
    model_name: str
    model_artifact: str
    backend: str = "local"
