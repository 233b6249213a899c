"""HTTP serving of Nori predictions on this framework (a self-hosted B200 endpoint).

The request / response contract is the hosted Nori API's (reference
``libs/synthefy/src/synthefy/data_models.py:20-175``), so ``SynthefyNoriClient(mode=
"remote", base_url=...)`` talks to either: ``POST /predict`` with JSON ``{"X_train":
[[...]], "y_train": [...], "X_test": [[...]], "task": "regression"}`` plus the optional
``model``, ``output_type``, ``quantiles``, ``discretize``, ``categorical_levels``,
``memory_policy``, ``large_context_policy`` / ``large_context_threshold``; missing
feature values are JSON ``null``.  The response is ``{"task", "predictions": [...]}``
with ``"quantiles"`` (one list per requested level) for ``output_type="quantiles"`` and
``"quantiles"`` / ``"taus"`` / ``"mean"`` for ``"full"``.

Models are loaded once per name and kept on the GPU; requests run one at a time per
process (the GPU is the serialisation point).  Run with
``python -m synthefy_nori_b200.serving --host 127.0.0.1 --port 8000 --weights random``.
"""

from __future__ import annotations

import argparse
import threading

import numpy as np
from starlette.requests import Request

from synthefy_nori_b200.client.data_models import MemoryReport, NoriPredictOptions, NoriPredictRequest
from synthefy_nori_b200.client.sagemaker import CONTENT_TYPE as TENSORFILE_CONTENT_TYPE

_LOCK = threading.Lock()
PredictRequest = NoriPredictRequest  # the request body model (validated on arrival)


def _matrix(rows) -> np.ndarray:
    return np.array([[np.nan if v is None else float(v) for v in r] for r in rows], dtype=np.float32)


def _options(req) -> dict:
    return {k: getattr(req, k) for k in NoriPredictOptions.model_fields}


def create_app(*, default_model: str = "nori-6m", weights: str | None = None, device=None, api_key: str | None = None,
               model_paths: dict | None = None):
    """``model_paths`` maps extra model names (fine-tuned checkpoints) to local files.

    Routes: ``POST /predict`` (the hosted JSON contract, bearer key when ``api_key`` is set),
    and the SageMaker container contract, ``GET /ping`` and ``POST /invocations``, which
    takes either the JSON body or a request tensor file
    (``application/vnd.synthefy.nori.tensorfile``, see ``client.sagemaker``) - what an
    asynchronous endpoint forwards from its S3 input location."""
    from fastapi import FastAPI, Header, HTTPException

    from synthefy_nori_b200.api import NoriRegressor

    app = FastAPI(title="Nori (B200)")
    models: dict = {}

    def run(opts: dict, Xtr: np.ndarray, y: np.ndarray, Xte: np.ndarray) -> dict:
        name = opts.get("model") or default_model
        paths = model_paths or {}
        kw = dict(model=name if name not in paths else None, model_path=paths.get(name),
                  weights=None if name in paths else weights, device=device, memory_policy=opts.get("memory_policy"),
                  large_context_policy=opts.get("large_context_policy"),
                  large_context_threshold=opts.get("large_context_threshold"),
                  random_state=opts.get("large_context_seed") or 0)
        if opts.get("multi_target_prediction_strategy"):
            kw["multi_target_prediction_strategy"] = opts["multi_target_prediction_strategy"]
        if opts.get("multi_target_prediction_policy"):
            kw["multi_target_prediction_policy"] = opts["multi_target_prediction_policy"]
        ot = opts.get("output_type") or "mean"
        task = opts.get("task") or "regression"
        try:
            with _LOCK:
                reg = NoriRegressor(**kw)
                if name in models:
                    reg._model_obj = models[name]
                reg.fit(Xtr, y)
                models[name] = reg._load_model()
                if opts.get("discretize") is not None or opts.get("categorical_levels") is not None:
                    out = reg.predict(Xte, discretize=opts.get("discretize"),
                                      categorical_levels=opts.get("categorical_levels"))
                    return {"task": task, "model": name, "predictions": np.asarray(out, float).tolist()}
                if ot == "full":
                    d = reg.predict(Xte, output_type="full")
                    return {"task": task, "model": name, "predictions": d["mean"].tolist(),
                            "mean": d["mean"].tolist(), "quantiles": d["quantiles"].tolist(),
                            "taus": d["taus"].tolist()}
                if ot == "quantiles":
                    q = reg.predict(Xte, output_type="quantiles", quantiles=opts.get("quantiles"))
                    med = reg.predict(Xte, output_type="median")
                    return {"task": task, "model": name, "predictions": med.tolist(), "quantiles": q.tolist()}
                out = reg.predict(Xte, output_type=ot)
                rep = MemoryReport.from_policy(getattr(reg, "memory_policy_", None)).model_dump()
                return {"task": task, "predictions": np.asarray(out, float).tolist(), "model": name,
                        "output_type": ot, "memory_report": rep}
        except (ValueError, NotImplementedError) as exc:
            raise HTTPException(status_code=422, detail=str(exc)) from exc

    def run_json(req: NoriPredictRequest) -> dict:
        return run(_options(req), _matrix(req.X_train), np.asarray(req.y_train, np.float64), _matrix(req.X_test))

    @app.get("/health")
    def health():
        return {"status": "ok", "models": sorted(models)}

    @app.get("/ping")
    def ping():
        return {"status": "ok"}

    @app.post("/predict")
    def predict(req: PredictRequest, authorization: str | None = Header(default=None)):
        if api_key is not None and authorization != f"Bearer {api_key}":
            raise HTTPException(status_code=401, detail="invalid API key")
        return run_json(req)

    @app.post("/invocations")
    async def invocations(request: Request):
        body = await request.body()
        ctype = (request.headers.get("content-type") or "").split(";")[0].strip()
        if ctype == TENSORFILE_CONTENT_TYPE:
            try:
                arrays, opts = tensorfile_request(body)
            except ValueError as exc:
                raise HTTPException(status_code=422, detail=str(exc)) from exc
            return run(opts, arrays["X_train"], arrays["y_train"], arrays["X_test"])
        try:
            req = NoriPredictRequest.model_validate_json(body)
        except ValueError as exc:
            raise HTTPException(status_code=422, detail=str(exc)) from exc
        return run_json(req)

    return app


def tensorfile_request(body: bytes) -> tuple[dict, dict]:
    """Arrays and validated options of a request tensor file given as bytes."""
    import os
    import tempfile

    from synthefy_nori_b200.client.sagemaker import read_tensorfile

    fd, path = tempfile.mkstemp(suffix=".tensorfile")
    try:
        with os.fdopen(fd, "wb") as f:
            f.write(body)
        arrays, meta = read_tensorfile(path)
    finally:
        os.unlink(path)
    opts = NoriPredictOptions.model_validate(meta)
    n, f = arrays["X_train"].shape if arrays["X_train"].ndim == 2 else (0, 0)
    if n == 0 or arrays["X_test"].ndim != 2 or arrays["X_test"].shape[0] == 0 or arrays["X_test"].shape[1] != f:
        raise ValueError("X_train and X_test must be non-empty matrices with the same number of features")
    if arrays["y_train"].shape[0] != n:
        raise ValueError("y_train must have one entry per X_train row")
    return arrays, _options(opts)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Serve Nori predictions over HTTP")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--model", default="nori-6m")
    ap.add_argument("--weights", default=None, help="'random' for random-init weights (no download)")
    ap.add_argument("--device", default=None)
    ap.add_argument("--api-key", default=None)
    a = ap.parse_args(argv)
    import uvicorn

    uvicorn.run(create_app(default_model=a.model, weights=a.weights, device=a.device, api_key=a.api_key),
                host=a.host, port=a.port)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
