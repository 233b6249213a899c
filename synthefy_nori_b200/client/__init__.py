"""Client SDK (reference ``libs/synthefy/src/synthefy/nori_client.py:1135-2937``).

``SynthefyNoriClient(mode="local", model=...)`` runs predictions in-process on this
framework.  ``mode="remote"`` POSTs the hosted API's JSON contract (see
``synthefy_nori_b200.serving``) to ``base_url + endpoint`` with ``Authorization:
<scheme> <api_key>``; responses 408 / 409 / 425 / 429 / 5xx and connection errors are
retried up to ``max_retries`` times, waiting ``Retry-After`` seconds when the server sends
it, else ``min(2^attempt, 30) * U[0.5, 1]`` seconds.  NaN features travel as ``null``;
non-finite targets are rejected before sending.  ``mode="sagemaker"`` runs S3-staged
asynchronous invocations of a SageMaker endpoint (``client.sagemaker``): its AWS clients
come from ``boto3`` (standard credential chain) or are passed in as
``sagemaker_runtime_client=`` / ``s3_client=``.
"""

from __future__ import annotations

import json
import os
import random
import time

import numpy as np

from synthefy_nori_b200.api import NoriRegressor

DEFAULT_BASE_URL = "https://inference.baseten.co"
DEFAULT_ENDPOINT = "/predict"
RETRY_STATUS = (408, 409, 425, 429)


class APIError(RuntimeError):
    def __init__(self, message: str, status_code: int | None = None):
        super().__init__(message)
        self.status_code = status_code


class APIConnectionError(APIError):
    pass


class APITimeoutError(APIConnectionError):
    pass


def _rows(a) -> list:
    a = np.asarray(a.to_numpy() if hasattr(a, "to_numpy") else a, np.float64)
    if a.ndim == 1:
        a = a[:, None]
    return [[None if not np.isfinite(v) else float(v) for v in r] for r in a]


class SynthefyNoriClient:
    def __init__(self, api_key: str | None = None, *, mode: str = "local", model: str | None = None,
                 model_path: str | None = None, weights: str | None = None, device=None, base_url: str | None = None,
                 endpoint: str = DEFAULT_ENDPOINT, timeout: float = 300.0, max_retries: int = 2,
                 auth_scheme: str = "Bearer", endpoint_name: str | None = None, region_name: str | None = None,
                 s3_staging_uri: str | None = None, sagemaker_runtime_client=None, s3_client=None,
                 **regressor_kwargs):
        if mode not in ("local", "remote", "sagemaker"):
            raise ValueError(f"mode must be 'local', 'remote' or 'sagemaker'; got {mode!r}")
        if model is None and model_path is None:
            raise ValueError("model is required (e.g. 'nori-6m'); there is no default")
        if timeout <= 0 or max_retries < 0:
            raise ValueError("timeout must be > 0 and max_retries >= 0")
        self.mode, self.model = mode, model
        self.timeout, self.max_retries = float(timeout), int(max_retries)
        if mode == "local":
            self._kw = dict(model=model, model_path=model_path, weights=weights, device=device, **regressor_kwargs)
        elif mode == "remote":
            import httpx

            self.api_key = api_key or os.environ.get("SYNTHEFY_API_KEY")
            if not self.api_key:
                raise ValueError("remote mode needs api_key= or SYNTHEFY_API_KEY")
            self.base_url = base_url or DEFAULT_BASE_URL
            self.endpoint, self.auth_scheme = endpoint, auth_scheme
            self.http = httpx.Client(base_url=self.base_url)
        else:
            from synthefy_nori_b200.client.sagemaker import SageMakerTransport

            if not endpoint_name or not s3_staging_uri:
                raise ValueError("mode='sagemaker' needs endpoint_name= and s3_staging_uri=")
            self.endpoint_name = endpoint_name
            self.sagemaker = SageMakerTransport(endpoint_name, s3_staging_uri, runtime_client=sagemaker_runtime_client,
                                                s3_client=s3_client, region_name=region_name, timeout=timeout)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def close(self) -> None:
        if getattr(self, "http", None) is not None:
            self.http.close()
            self.http = None

    # ------------------------------------------------------------------ predict
    def predict(self, X_train, y_train, X_test, *, output_type: str = "mean", quantiles=None, discretize=None,
                categorical_levels=None, memory_policy=None, large_context_policy=None,
                large_context_threshold=None):
        if self.mode == "sagemaker":
            return self._predict_sagemaker(X_train, y_train, X_test, output_type=output_type, quantiles=quantiles,
                                           discretize=discretize, categorical_levels=categorical_levels,
                                           memory_policy=memory_policy, large_context_policy=large_context_policy,
                                           large_context_threshold=large_context_threshold)
        if self.mode == "remote":
            return self._predict_remote(X_train, y_train, X_test, output_type=output_type, quantiles=quantiles,
                                        discretize=discretize, categorical_levels=categorical_levels,
                                        memory_policy=memory_policy, large_context_policy=large_context_policy,
                                        large_context_threshold=large_context_threshold)
        y = np.asarray(y_train)
        kw = dict(self._kw)
        if memory_policy is not None:
            kw["memory_policy"] = memory_policy
        if large_context_policy is not None:
            kw.update(large_context_policy=large_context_policy, large_context_threshold=large_context_threshold)
        reg = NoriRegressor(**kw).fit(X_train, y)
        if discretize is not None or categorical_levels is not None:
            return reg.predict(X_test, discretize=discretize, categorical_levels=categorical_levels)
        return reg.predict(X_test, output_type=output_type, quantiles=quantiles)

    # ------------------------------------------------------------------ remote
    def _payload(self, X_train, y_train, X_test, **opt) -> dict:
        y = np.asarray(y_train, np.float64)
        if not np.all(np.isfinite(y)):
            raise ValueError("y_train must contain only finite numbers for remote inference")
        p = {"X_train": _rows(X_train), "y_train": y.tolist(), "X_test": _rows(X_test), "task": "regression",
             "model": self.model}
        if opt.get("output_type") not in (None, "mean"):
            p["output_type"] = opt["output_type"]
        for k in ("quantiles", "discretize", "categorical_levels", "memory_policy", "large_context_policy",
                  "large_context_threshold"):
            if opt.get(k) is not None:
                v = opt[k]
                p[k] = v.model_dump(exclude_unset=True) if hasattr(v, "model_dump") else v
        return p

    def _backoff(self, attempt: int, response) -> float:
        if response is not None:
            ra = response.headers.get("retry-after")
            if ra is not None:
                try:
                    v = float(ra)
                    if np.isfinite(v):
                        return max(0.0, v)
                except ValueError:
                    pass
        return min(2 ** attempt, 30) * (0.5 + 0.5 * random.random())

    def _post(self, payload: dict):
        import httpx

        body = json.dumps(payload, allow_nan=False).encode()
        headers = {"Content-Type": "application/json", "Authorization": f"{self.auth_scheme} {self.api_key}",
                   "User-Agent": "synthefy-nori-b200"}
        for attempt in range(self.max_retries + 1):
            resp, err = None, None
            try:
                resp = self.http.post(self.endpoint, content=body, headers=headers, timeout=self.timeout)
                if resp.status_code < 400:
                    return resp.json()
                retry = resp.status_code in RETRY_STATUS or resp.status_code >= 500
                if not retry:
                    raise APIError(f"HTTP {resp.status_code}: {resp.text[:500]}", resp.status_code)
            except httpx.TimeoutException as exc:
                err = APITimeoutError(str(exc))
            except httpx.HTTPError as exc:
                err = APIConnectionError(str(exc))
            if attempt < self.max_retries:
                time.sleep(self._backoff(attempt, resp))
                continue
            if err is not None:
                raise err
            raise APIError(f"HTTP {resp.status_code}: {resp.text[:500]}", resp.status_code)
        raise APIConnectionError("request failed after retries")

    def _predict_remote(self, X_train, y_train, X_test, **opt):
        return self._parse(self._post(self._payload(X_train, y_train, X_test, **opt)), opt)

    # ------------------------------------------------------------------ SageMaker
    def _predict_sagemaker(self, X_train, y_train, X_test, **opt):
        """One S3-staged asynchronous invocation of the endpoint (``client.sagemaker``): the
        arrays travel in a request tensor file, the options in its metadata."""
        y = np.asarray(y_train, np.float64)
        if not np.all(np.isfinite(y)):
            raise ValueError("y_train must contain only finite numbers for hosted inference")

        def mat(a):
            a = np.asarray(a.to_numpy() if hasattr(a, "to_numpy") else a, np.float32)
            return a[:, None] if a.ndim == 1 else a

        meta = {"task": "regression"}
        if opt.get("output_type") not in (None, "mean"):
            meta["output_type"] = opt["output_type"]
        for k in ("quantiles", "discretize", "categorical_levels", "memory_policy", "large_context_policy",
                  "large_context_threshold"):
            if opt.get(k) is not None:
                v = opt[k]
                v = v.model_dump(exclude_unset=True) if hasattr(v, "model_dump") else v
                meta[k] = v.tolist() if isinstance(v, np.ndarray) else v
        data = self.sagemaker.invoke({"X_train": mat(X_train), "y_train": y, "X_test": mat(X_test)}, meta,
                                     model=self.model)
        return self._parse(data, opt)

    @staticmethod
    def _parse(data: dict, opt: dict):
        ot = opt.get("output_type") or "mean"
        if ot == "full":
            return {"quantiles": np.asarray(data["quantiles"], float), "taus": np.asarray(data["taus"], float),
                    "mean": np.asarray(data["mean"], float)}
        if ot == "quantiles":
            return np.asarray(data["quantiles"], float)
        return np.array([np.nan if v is None else v for v in data["predictions"]], float)


from synthefy_nori_b200.client.sagemaker import SageMakerInvocationError  # noqa: E402

__all__ = ["SynthefyNoriClient", "APIError", "APIConnectionError", "APITimeoutError", "SageMakerInvocationError"]
