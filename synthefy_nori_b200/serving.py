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

from synthefy_nori_b200.client.data_models import MemoryReport, NoriPredictRequest

_LOCK = threading.Lock()
PredictRequest = NoriPredictRequest  # the request body model (validated on arrival)


def _matrix(rows) -> np.ndarray:
    return np.array([[np.nan if v is None else float(v) for v in r] for r in rows], dtype=np.float32)


def create_app(*, default_model: str = "nori-6m", weights: str | None = None, device=None, api_key: str | None = None,
               model_paths: dict | None = None):
    """``model_paths`` maps extra model names (fine-tuned checkpoints) to local files."""
    from fastapi import FastAPI, Header, HTTPException

    from synthefy_nori_b200.api import NoriRegressor

    app = FastAPI(title="Nori (B200)")
    models: dict = {}

    @app.get("/health")
    def health():
        return {"status": "ok", "models": sorted(models)}

    @app.post("/predict")
    def predict(req: PredictRequest, authorization: str | None = Header(default=None)):
        if api_key is not None and authorization != f"Bearer {api_key}":
            raise HTTPException(status_code=401, detail="invalid API key")
        if req.task != "regression":
            raise HTTPException(status_code=422, detail="only task='regression' is supported")
        name = req.model or default_model
        Xtr, Xte = _matrix(req.X_train), _matrix(req.X_test)
        y = np.asarray(req.y_train, np.float64)
        paths = model_paths or {}
        kw = dict(model=name if name not in paths else None, model_path=paths.get(name),
                  weights=None if name in paths else weights, device=device, memory_policy=req.memory_policy,
                  large_context_policy=req.large_context_policy, large_context_threshold=req.large_context_threshold,
                  random_state=req.large_context_seed or 0)
        if req.multi_target_prediction_strategy:
            kw["multi_target_prediction_strategy"] = req.multi_target_prediction_strategy
        if req.multi_target_prediction_policy:
            kw["multi_target_prediction_policy"] = req.multi_target_prediction_policy
        ot = req.output_type or "mean"
        try:
            with _LOCK:
                reg = NoriRegressor(**kw)
                if name in models:
                    reg._model_obj = models[name]
                reg.fit(Xtr, y)
                models[name] = reg._load_model()
                if req.discretize is not None or req.categorical_levels is not None:
                    out = reg.predict(Xte, discretize=req.discretize, categorical_levels=req.categorical_levels)
                    return {"task": req.task, "predictions": np.asarray(out, float).tolist()}
                if ot == "full":
                    d = reg.predict(Xte, output_type="full")
                    return {"task": req.task, "predictions": d["mean"].tolist(), "mean": d["mean"].tolist(),
                            "quantiles": d["quantiles"].tolist(), "taus": d["taus"].tolist()}
                if ot == "quantiles":
                    q = reg.predict(Xte, output_type="quantiles", quantiles=req.quantiles)
                    med = reg.predict(Xte, output_type="median")
                    return {"task": req.task, "predictions": med.tolist(), "quantiles": q.tolist()}
                out = reg.predict(Xte, output_type=ot)
                rep = MemoryReport.from_policy(getattr(reg, "memory_policy_", None)).model_dump()
                return {"task": req.task, "predictions": np.asarray(out, float).tolist(), "model": name,
                        "output_type": ot, "memory_report": rep}
        except (ValueError, NotImplementedError) as exc:
            raise HTTPException(status_code=422, detail=str(exc)) from exc

    return app


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
