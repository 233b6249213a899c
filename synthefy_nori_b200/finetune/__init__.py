"""Fine-tune a released Nori model on your own tables, then serve it.

``SynthefyNoriFineTuner`` keeps the reference client's job API (``fine_tune``, ``wait``,
``get_status``, ``stop``, ``get_logs``, ``get_training_curves``, ``get_training_report``,
``get_training_plan``, ``deploy``, ``undeploy``, ``create_client``; reference
``libs/synthefy/src/synthefy/nori_fine_tune.py``) with two backends:

* ``backend="local"`` (this build's): the job runs on this machine's GPU in a background
  thread.  The table (CSV / Parquet file or folder; optional task column: one model
  learns every task, episodes are drawn per task) is featurised like ``predict`` does,
  split into train / validation rows, and each of ``bag`` models (row partitions of the
  train split) is trained for ``n_steps_per_model`` optimizer steps on in-context
  episodes: random context rows + query rows from its partition (rows after the context
  in time order when a time column is given), the target standardised on the context,
  the 999-quantile pinball objective, AdamW + EMA on the native trainer.  The
  validation MSE (validation rows predicted from training-row context) is tracked every
  ``validation_every_n_steps`` steps with early stopping (``patience``); the best
  weights are written to ``output_path/<model_name>.pt`` in the release checkpoint
  format.  ``deploy`` starts this build's HTTP server (``serving.py``) with the
  fine-tuned model registered under its name;
* ``backend="sagemaker"``: hosted jobs run by the Nori Algorithm and asynchronous
  SageMaker endpoints (``finetune.sagemaker``); its AWS clients come from ``boto3`` or are
  passed in (``sagemaker_client=``, ``s3_client=``, ``logs_client=``).
"""

from __future__ import annotations

import glob
import os
import threading
import time
import uuid

import numpy as np
import torch

from synthefy_nori_b200.client.data_models import (ChildCurve, FineTunedEndpoint, FineTuneHyperparameters, FineTuneJob,
                                                   FineTuneJobRequest, TaskScore, TrainingPlan, TrainingReport)

__all__ = ["SynthefyNoriFineTuner", "FineTuneHyperparameters", "FineTuneJobRequest", "FineTuneJob", "TrainingReport",
           "TrainingPlan", "FineTunedEndpoint", "FineTuningError"]


class FineTuningError(RuntimeError):
    pass


def _read_table(path: str):
    import pandas as pd

    files = [path] if os.path.isfile(path) else sorted(glob.glob(os.path.join(path, "**", "*.*"), recursive=True))
    files = [f for f in files if f.endswith((".csv", ".parquet", ".pq"))]
    if not files:
        raise FineTuningError(f"no CSV or Parquet files under {path!r}")
    parts = [pd.read_parquet(f) if f.endswith((".parquet", ".pq")) else pd.read_csv(f) for f in files]
    return pd.concat(parts, ignore_index=True)


def _rows_draw(spec, rng, default: int, cap: int) -> int:
    if spec is None:
        n = default
    elif isinstance(spec, int):
        n = spec
    else:
        keys = [int(k) for k in spec]
        w = np.asarray([float(spec[k]) for k in spec], np.float64)
        n = keys[int(rng.choice(len(keys), p=w / w.sum()))]
    return max(1, min(int(n), cap))


class _LocalJob:
    def __init__(self, req: FineTuneJobRequest, device):
        self.req = req
        self.hp = req.hyperparameters
        self.device = torch.device(device)
        self.name = req.job_name or f"{self.hp.model_name}-{uuid.uuid4().hex[:8]}"
        self.job = FineTuneJob(job_name=self.name, status="Pending", created_at=time.time(), model_name=self.hp.model_name)
        self.logs: list[str] = []
        self.report = TrainingReport()
        self.plan: TrainingPlan | None = None
        self._stop = threading.Event()
        self.thread = threading.Thread(target=self._run, name=f"finetune-{self.name}", daemon=True)

    def log(self, msg: str) -> None:
        self.logs.append(f"[{time.strftime('%H:%M:%S')}] {msg}")

    # ---------------------------------------------------------------- data
    def _prepare(self):
        from synthefy_nori_b200.featurize import DataFramePreprocessor

        hp = self.hp
        df = _read_table(self.req.training_data)
        if hp.target_column not in df:
            raise FineTuningError(f"target column {hp.target_column!r} not in the table")
        drop = {hp.target_column} | {c for c in (hp.task_column, hp.time_column) if c}
        feats = hp.feature_columns or [c for c in df.columns if c not in drop]
        if hp.time_column:
            df = df.sort_values(hp.time_column, kind="stable").reset_index(drop=True)
        y = df[hp.target_column].to_numpy(np.float64)
        ok = np.isfinite(y)
        df, y = df[ok].reset_index(drop=True), y[ok]
        pre = DataFramePreprocessor()
        X = pre.fit_transform(df[feats]).to_numpy(np.float32)
        tasks = df[hp.task_column].astype(str).to_numpy() if hp.task_column else np.zeros(len(df), dtype=object)
        return X, y.astype(np.float32), tasks, pre, feats

    def _split(self, n_rows_task: np.ndarray, rng):
        """Train / validation rows (the latest rows of each task when time-ordered)."""
        hp = self.hp
        idx = np.arange(len(n_rows_task))
        val = []
        for t in np.unique(n_rows_task):
            rows = idx[n_rows_task == t]
            k = max(1, int(round(len(rows) * hp.validation_fraction)))
            val.append(rows[-k:] if hp.time_column else rng.choice(rows, k, replace=False))
        val = np.sort(np.concatenate(val))
        train = np.setdiff1d(idx, val)
        return train, val

    # ---------------------------------------------------------------- training
    def _episode(self, X, y, rows, rng, n_ctx, n_q):
        if self.hp.time_column:
            start = int(rng.integers(0, max(1, len(rows) - n_ctx - n_q) + 1))
            sel = rows[start : start + n_ctx + n_q]
        else:
            sel = rng.choice(rows, min(len(rows), n_ctx + n_q), replace=False)
        xe, ye = X[sel], y[sel].astype(np.float64)
        c = min(n_ctx, len(sel) - 1)
        mu, sd = ye[:c].mean(), ye[:c].std() or 1.0
        return xe, ((ye - mu) / sd).astype(np.float32), c

    def _val_mse(self, model, X, y, train, val, rng):
        from synthefy_nori_b200.api import NoriRegressor

        ctx = train if len(train) <= 4096 else rng.choice(train, 4096, replace=False)
        reg = NoriRegressor(model=None, n_estimators=1, device=self.device)
        reg._model_obj = model
        reg.fit(X[ctx], y[ctx])
        pred = reg.predict(X[val])
        return float(np.mean((pred - y[val]) ** 2))

    def _run(self):
        from synthefy_nori_b200.models.config import preset_config
        from synthefy_nori_b200.training.trainer import NoriTrainer, TrainConfig
        from synthefy_nori_b200.utils.loading import build_model, load_model, save_release_checkpoint

        hp = self.hp
        self.job.status = "InProgress"
        t_end = time.time() + hp.max_training_hours * 3600 if hp.max_training_hours else None
        try:
            rng = np.random.default_rng(hp.seed)
            X, y, tasks, _pre, feats = self._prepare()
            train, val = self._split(tasks, rng)
            n_ctx = _rows_draw(hp.context_rows, rng, min(1024, max(16, len(train) // 2)), max(1, len(train) - 1))
            n_q = _rows_draw(hp.query_rows, rng, min(1024, max(1, len(train) - n_ctx)), max(1, len(train) - n_ctx))
            self.plan = TrainingPlan(n_models=hp.bag, n_train_rows=len(train), n_val_rows=len(val),
                                     n_features=X.shape[1], steps_per_model=hp.n_steps_per_model, context_rows=n_ctx,
                                     query_rows=n_q)
            self.log(f"plan: {self.plan.model_dump()}")
            if hp.weights == "random":
                base = build_model(preset_config(hp.base_model))
                torch.manual_seed(hp.seed)
            else:
                from synthefy_nori_b200.hf import download_checkpoint

                base = load_model(hp.base_model if os.path.isfile(hp.base_model) else download_checkpoint(hp.base_model))
            config = dict(getattr(base, "model_config", None) or preset_config(hp.base_model))
            before = self._val_mse(base.to(self.device), X, y, train, val, rng)
            self.report.val_mse_before = before
            self.log(f"validation MSE before: {before:.6g}")
            parts = np.array_split(rng.permutation(train), hp.bag)
            states, best_mses = [], []
            for mi, part in enumerate(parts):
                model = build_model(dict(config))
                model.load_state_dict(base.state_dict())
                tr = NoriTrainer(model, TrainConfig(lr=hp.lr, ema_decay=None, loss_spike_factor=None), self.device)
                curve = ChildCurve(model_index=mi)
                best, best_state, best_step, bad = float("inf"), None, 0, 0
                rows = np.sort(part) if hp.time_column else part
                for step in range(1, hp.n_steps_per_model + 1):
                    if self._stop.is_set() or (t_end is not None and time.time() > t_end):
                        self.report.stopped_early = True
                        break
                    eps = [self._episode(X, y, rows, rng, n_ctx, n_q) for _ in range(hp.batch_size)]
                    c = min(e[2] for e in eps)
                    n = min(len(e[0]) for e in eps)
                    xb = torch.from_numpy(np.stack([e[0][:n] for e in eps])).to(self.device)
                    yb = torch.from_numpy(np.stack([e[1][:n] for e in eps])).to(self.device)
                    loss = float(tr.train_step(torch.nan_to_num(xb, nan=float("nan")), yb, c))
                    curve.steps.append(step)
                    curve.train_loss.append(loss)
                    if step % hp.validation_every_n_steps == 0 or step == hp.n_steps_per_model:
                        model.eval()
                        mse = self._val_mse(model, X, y, rows, val, rng)
                        model.train()
                        curve.val_mse.append(mse)
                        self.log(f"model {mi} step {step}: loss {loss:.5g} val MSE {mse:.6g}")
                        if mse < best:
                            best, best_step, bad = mse, step, 0
                            best_state = {k: v.detach().cpu().clone() for k, v in model.state_dict().items()}
                        else:
                            bad += 1
                            if hp.patience is not None and bad >= hp.patience:
                                self.report.stopped_early = True
                                break
                tr.close()
                states.append(best_state or {k: v.detach().cpu() for k, v in model.state_dict().items()})
                best_mses.append(best)
                self.report.curves.append(curve)
                self.report.best_step.append(best_step)
            # the bag's average weights are the fine-tuned model
            avg = {k: sum(s[k].float() for s in states) / len(states) if states[0][k].is_floating_point()
                   else states[0][k] for k in states[0]}
            final = build_model(dict(config))
            final.load_state_dict(avg)
            after = self._val_mse(final.to(self.device), X, y, train, val, rng)
            self.report.val_mse_after = after
            if self.hp.task_column:
                for t in np.unique(tasks):
                    self.report.task_scores.append(TaskScore(task=str(t), val_mse_before=before, val_mse_after=after))
            os.makedirs(self.req.output_path, exist_ok=True)
            out = os.path.join(self.req.output_path, f"{hp.model_name}.pt")
            save_release_checkpoint(final.cpu(), config, out)
            self.job.model_artifact = out
            self.log(f"validation MSE after: {after:.6g}; wrote {out}")
            self.job.status = "Stopped" if self._stop.is_set() else "Completed"
        except Exception as exc:  # noqa: BLE001 - reported through the job status
            self.job.status = "Failed"
            self.job.failure_reason = f"{type(exc).__name__}: {exc}"
            self.log(f"failed: {self.job.failure_reason}")
        finally:
            self.job.ended_at = time.time()


class SynthefyNoriFineTuner:
    """Fine-tuning jobs and the endpoints serving their results."""

    def __init__(self, *, backend: str = "local", device=None, region_name: str | None = None,
                 sagemaker_client=None, s3_client=None, logs_client=None, poll_s: float = 15.0):
        if backend not in ("local", "sagemaker"):
            raise ValueError("backend must be 'local' or 'sagemaker'")
        self.backend = backend
        self.device = device or ("cuda" if torch.cuda.is_available() else "cpu")
        self.region_name = region_name
        self._jobs: dict[str, _LocalJob] = {}
        self._servers: dict[str, tuple] = {}
        self._sm = None
        if backend == "sagemaker":
            from synthefy_nori_b200.finetune.sagemaker import SageMakerJobs

            self._sm = SageMakerJobs(region_name=region_name, sagemaker_client=sagemaker_client, s3_client=s3_client,
                                     logs_client=logs_client, poll_s=poll_s)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def close(self) -> None:
        for name in list(self._servers):
            self.undeploy(name)

    # ---------------------------------------------------------------- jobs
    def get_training_plan(self, request: FineTuneJobRequest) -> TrainingPlan:
        job = _LocalJob(request, self.device)
        X, y, tasks, _, _ = job._prepare()
        rng = np.random.default_rng(request.hyperparameters.seed)
        train, val = job._split(tasks, rng)
        hp = request.hyperparameters
        n_ctx = _rows_draw(hp.context_rows, rng, min(1024, max(16, len(train) // 2)), max(1, len(train) - 1))
        n_q = _rows_draw(hp.query_rows, rng, min(1024, max(1, len(train) - n_ctx)), max(1, len(train) - n_ctx))
        return TrainingPlan(n_models=hp.bag, n_train_rows=len(train), n_val_rows=len(val), n_features=X.shape[1],
                            steps_per_model=hp.n_steps_per_model, context_rows=n_ctx, query_rows=n_q)

    def fine_tune(self, request: FineTuneJobRequest, *, overwrite: bool = False) -> FineTuneJob:
        if self._sm is not None:
            return self._sm.fine_tune(request)
        out = os.path.join(request.output_path, f"{request.hyperparameters.model_name}.pt")
        if os.path.exists(out) and not overwrite:
            raise FineTuningError(f"{out} exists; pass overwrite=True to replace it")
        job = _LocalJob(request, self.device)
        self._jobs[job.name] = job
        job.thread.start()
        return job.job

    def _get(self, job_name: str) -> _LocalJob:
        if job_name not in self._jobs:
            raise KeyError(f"unknown job {job_name!r}")
        return self._jobs[job_name]

    def get_status(self, job_name: str) -> FineTuneJob:
        if self._sm is not None:
            return self._sm.get_status(job_name)
        return self._get(job_name).job

    def wait(self, job_name: str, *, poll_s: float = 1.0, timeout_s: float | None = None) -> FineTuneJob:
        if self._sm is not None:
            return self._sm.wait(job_name, poll_s=poll_s, timeout_s=timeout_s)
        j = self._get(job_name)
        j.thread.join(timeout_s)
        if j.thread.is_alive():
            raise TimeoutError(f"job {job_name} still running after {timeout_s} s")
        return j.job

    def stop(self, job_name: str) -> FineTuneJob:
        if self._sm is not None:
            return self._sm.stop(job_name)
        j = self._get(job_name)
        j._stop.set()
        if j.job.status == "InProgress":
            j.job.status = "Stopping"
        return j.job

    def get_logs(self, job_name: str, *, follow: bool = False, poll_s: float = 0.5):
        if self._sm is not None:
            yield from self._sm.get_logs(job_name, follow=follow, poll_s=poll_s)
            return
        j = self._get(job_name)
        i = 0
        while True:
            while i < len(j.logs):
                yield j.logs[i]
                i += 1
            if not follow or not j.thread.is_alive():
                while i < len(j.logs):
                    yield j.logs[i]
                    i += 1
                return
            time.sleep(poll_s)

    def get_training_curves(self, job_name: str) -> dict:
        r = self.get_training_report(job_name)
        return {f"model_{c.model_index}": c.model_dump() for c in r.curves}

    def get_training_report(self, job_name: str) -> TrainingReport:
        if self._sm is not None:
            return self._sm.get_training_report(job_name)
        return self._get(job_name).report

    # ---------------------------------------------------------------- serving
    def deploy(self, job: FineTuneJob | str, *, host: str = "127.0.0.1", port: int = 0, **sagemaker_kw) -> FineTunedEndpoint:
        """Serve a completed job's model: this build's HTTP server (local backend) or an
        asynchronous SageMaker endpoint (``endpoint_name=``, ``instance_type=``; sagemaker)."""
        if self._sm is not None:
            return self._sm.deploy(job if isinstance(job, str) else job.job_name, **sagemaker_kw)
        j = self._get(job if isinstance(job, str) else job.job_name)
        if j.job.status != "Completed" or not j.job.model_artifact:
            raise FineTuningError(f"job {j.name} has no completed model to deploy (status {j.job.status})")
        import socket

        import uvicorn

        from synthefy_nori_b200.serving import create_app

        if port == 0:
            s = socket.socket()
            s.bind((host, 0))
            port = s.getsockname()[1]
            s.close()
        app = create_app(default_model=j.hp.model_name, device=self.device,
                         model_paths={j.hp.model_name: j.job.model_artifact})
        server = uvicorn.Server(uvicorn.Config(app, host=host, port=port, log_level="warning"))
        th = threading.Thread(target=server.run, daemon=True)
        th.start()
        t0 = time.time()
        while not server.started and time.time() - t0 < 30:
            time.sleep(0.05)
        name = f"{j.hp.model_name}-endpoint"
        self._servers[name] = (server, th)
        return FineTunedEndpoint(endpoint_name=name, url=f"http://{host}:{port}", model_name=j.hp.model_name,
                                 model_artifact=j.job.model_artifact)

    def undeploy(self, endpoint: FineTunedEndpoint | str, *, timeout_s: float = 30.0) -> None:
        name = endpoint if isinstance(endpoint, str) else endpoint.endpoint_name
        if self._sm is not None:
            self._sm.undeploy(name)
            return
        srv = self._servers.pop(name, None)
        if srv is None:
            return
        server, th = srv
        server.should_exit = True
        th.join(timeout_s)

    def create_client(self, endpoint: FineTunedEndpoint, **kw):
        from synthefy_nori_b200.client import SynthefyNoriClient

        if endpoint.backend == "sagemaker":
            if self._sm is None:
                raise FineTuningError("a SageMaker endpoint needs a tuner with backend='sagemaker'")
            staging = kw.pop("s3_staging_uri", None) or self._sm.staging_uri(endpoint.endpoint_name)
            if staging is None:
                raise FineTuningError("pass s3_staging_uri= for an endpoint this tuner did not deploy")
            return SynthefyNoriClient(mode="sagemaker", model=endpoint.model_name,
                                      endpoint_name=endpoint.endpoint_name, s3_staging_uri=staging,
                                      s3_client=kw.pop("s3_client", self._sm.s3), region_name=self.region_name, **kw)
        return SynthefyNoriClient(api_key=kw.pop("api_key", "local"), mode="remote", model=endpoint.model_name,
                                  base_url=endpoint.url, **kw)
