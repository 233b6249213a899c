"""SageMaker asynchronous inference for ``SynthefyNoriClient(mode="sagemaker")``.

Reference: ``libs/synthefy/src/synthefy/nori_client.py:2464-2680`` (the S3-staged
``InvokeEndpointAsync`` flow) and ``nori_payload.py`` (the request tensor file).

One call:

1. the request is written as a tensor file (below) and uploaded to
   ``<s3_staging_uri>/<endpoint>/<invocation id>/request.tensorfile``;
2. ``InvokeEndpointAsync`` is called with that input location, the invocation id as
   ``InferenceId`` and an output path extension ``invocations/<invocation id>`` so the
   result and failure objects land in a prefix that belongs to this call alone (a response
   that points anywhere else is refused);
3. the failure and output objects are polled with ``HeadObject`` under exponential backoff
   with jitter until the client timeout; a failure object raises
   :class:`SageMakerInvocationError` carrying the endpoint's message;
4. the result JSON is read, its ``model`` checked against the requested model, and the
   staged objects deleted. When the call's fate is unknown (the invoke raised after the
   upload, or the wait timed out) the input is left for the bucket's lifecycle rule,
   because a queued invocation may still read it.

The AWS clients are any objects with boto3's method names (``upload_file``,
``head_object``, ``download_file``, ``delete_object``; ``invoke_endpoint_async``):
``boto3`` builds them when it is installed, and callers (and the tests) may pass their own.

Tensor file (the wire format the hosted container reads; it must stay byte-compatible):
an 8-byte magic ``NORI_REQ`` and a little-endian uint32 header length, the UTF-8 JSON
header ``{"format": "synthefy-nori-request-v1", "metadata": {...}, "tensors": {name:
{"dtype", "shape", "offset", "nbytes"}}}`` (sorted keys, compact separators), zero padding
to 64 KiB, then the raw little-endian arrays ``X_train`` (float32), ``y_train`` (float64),
``X_test`` (float32) at their offsets. NaN features travel as NaN inside the arrays.
"""

from __future__ import annotations

import json
import os
import random
import struct
import tempfile
import time
import uuid
import warnings

import numpy as np

CONTENT_TYPE = "application/vnd.synthefy.nori.tensorfile"
FORMAT_VERSION = "synthefy-nori-request-v1"
MAX_INPUT_BYTES = 1024 ** 3  # the asynchronous-inference payload limit
HEADER_BYTES = 64 * 1024
_MAGIC = b"NORI_REQ"
_PREFIX = struct.Struct("<8sI")
TENSOR_DTYPES = {"X_train": np.dtype("<f4"), "y_train": np.dtype("<f8"), "X_test": np.dtype("<f4")}
REQUEST_TTL_SECONDS = 6 * 3600
INVOCATION_TIMEOUT_SECONDS = 3600
POLL_INITIAL_SECONDS = 0.5
POLL_MAX_SECONDS = 10.0


class SageMakerInvocationError(RuntimeError):
    """The endpoint wrote a failure object for this invocation."""

    def __init__(self, message: str, *, invocation_id: str, failure_location: str | None):
        super().__init__(message)
        self.invocation_id = invocation_id
        self.failure_location = failure_location


# ---------------------------------------------------------------- tensor file
def write_tensorfile(path, arrays: dict, metadata: dict) -> int:
    """Write the request tensor file; returns its size in bytes."""
    tensors, blobs, offset = {}, [], HEADER_BYTES
    for name, dt in TENSOR_DTYPES.items():
        a = np.ascontiguousarray(arrays[name], dtype=dt)
        tensors[name] = {"dtype": a.dtype.str, "shape": list(a.shape), "offset": offset, "nbytes": int(a.nbytes)}
        blobs.append(a)
        offset += a.nbytes
    if offset > MAX_INPUT_BYTES:
        raise ValueError("the serialized request exceeds the 1 GB asynchronous-inference payload limit; "
                         "send fewer context or query rows")
    header = json.dumps({"format": FORMAT_VERSION, "metadata": metadata, "tensors": tensors},
                        separators=(",", ":"), sort_keys=True, allow_nan=False).encode("utf-8")
    if _PREFIX.size + len(header) > HEADER_BYTES:
        raise ValueError("request metadata does not fit the 64 KiB tensor-file header")
    with open(path, "wb") as f:
        f.write(_PREFIX.pack(_MAGIC, len(header)))
        f.write(header)
        f.write(bytes(HEADER_BYTES - _PREFIX.size - len(header)))
        for a in blobs:
            f.write(a.tobytes())
    return offset


def read_tensorfile(path) -> tuple[dict, dict]:
    """(arrays, metadata) of a request tensor file, checked against its header."""
    with open(path, "rb") as f:
        raw = f.read()
    if len(raw) < HEADER_BYTES:
        raise ValueError("tensor file shorter than its header")
    magic, n = _PREFIX.unpack_from(raw, 0)
    if magic != _MAGIC or n > HEADER_BYTES - _PREFIX.size:
        raise ValueError("not a Nori request tensor file")
    head = json.loads(raw[_PREFIX.size: _PREFIX.size + n].decode("utf-8"))
    if head.get("format") != FORMAT_VERSION:
        raise ValueError(f"unsupported tensor-file format {head.get('format')!r}")
    arrays = {}
    for name, dt in TENSOR_DTYPES.items():
        t = head["tensors"][name]
        if np.dtype(t["dtype"]) != dt:
            raise ValueError(f"{name}: dtype {t['dtype']} (expected {dt.str})")
        off, nb, shape = int(t["offset"]), int(t["nbytes"]), tuple(int(s) for s in t["shape"])
        if off < HEADER_BYTES or off + nb > len(raw) or nb != int(np.prod(shape, dtype=np.int64)) * dt.itemsize:
            raise ValueError(f"{name}: extent outside the file or inconsistent with its shape")
        arrays[name] = np.frombuffer(raw, dtype=dt, count=nb // dt.itemsize, offset=off).reshape(shape).copy()
    return arrays, dict(head.get("metadata") or {})


# ---------------------------------------------------------------- S3 helpers
def parse_s3_uri(uri: str) -> tuple[str, str]:
    if not isinstance(uri, str) or not uri.startswith("s3://"):
        raise ValueError(f"expected an s3://bucket/key URI, got {uri!r}")
    bucket, _, key = uri[5:].partition("/")
    if not bucket:
        raise ValueError(f"S3 URI without a bucket: {uri!r}")
    return bucket, key


def _missing(exc: Exception) -> bool:
    """Whether an S3 error means 'no such object' (boto3's ClientError 404 / NoSuchKey)."""
    resp = getattr(exc, "response", None)
    if isinstance(resp, dict):
        code = str((resp.get("Error") or {}).get("Code", ""))
        status = (resp.get("ResponseMetadata") or {}).get("HTTPStatusCode")
        return code in ("404", "NoSuchKey", "NotFound") or status == 404
    return isinstance(exc, (FileNotFoundError, KeyError))


def _owned(location: str | None, invocation_id: str) -> bool:
    if not location:
        return False
    try:
        _, key = parse_s3_uri(location)
    except ValueError:
        return False
    return f"/invocations/{invocation_id}/" in f"/{key}"


class SageMakerTransport:
    """Staged asynchronous invocations of one SageMaker endpoint."""

    def __init__(self, endpoint_name: str, s3_staging_uri: str, *, runtime_client=None, s3_client=None,
                 region_name: str | None = None, timeout: float = 300.0, poll_initial: float = POLL_INITIAL_SECONDS,
                 poll_max: float = POLL_MAX_SECONDS):
        if not endpoint_name:
            raise ValueError("endpoint_name is required")
        bucket, prefix = parse_s3_uri(s3_staging_uri)
        self.endpoint_name, self.bucket, self.prefix = endpoint_name, bucket, prefix.strip("/")
        if runtime_client is None or s3_client is None:
            try:
                import boto3
            except ImportError as exc:
                raise RuntimeError("mode='sagemaker' needs boto3 (or runtime_client= and s3_client=)") from exc
            session = boto3.Session(region_name=region_name)
            runtime_client = runtime_client or session.client("sagemaker-runtime")
            s3_client = s3_client or session.client("s3")
        self.runtime, self.s3 = runtime_client, s3_client
        self.timeout, self.poll_initial, self.poll_max = float(timeout), float(poll_initial), float(poll_max)

    def _exists(self, location: str) -> bool:
        bucket, key = parse_s3_uri(location)
        try:
            self.s3.head_object(Bucket=bucket, Key=key)
            return True
        except Exception as exc:  # noqa: BLE001
            if _missing(exc):
                return False
            raise

    def _read(self, location: str) -> str:
        bucket, key = parse_s3_uri(location)
        fd, path = tempfile.mkstemp(prefix="nori-result-", suffix=".json")
        os.close(fd)
        try:
            self.s3.download_file(bucket, key, path)
            with open(path, encoding="utf-8", errors="replace") as f:
                return f.read()
        finally:
            os.unlink(path)

    def _failure(self, location: str, invocation_id: str) -> SageMakerInvocationError:
        text = self._read(location)[:16384]
        msg = text.strip() or "SageMaker asynchronous inference failed"
        try:
            details = json.loads(text)
        except json.JSONDecodeError:
            details = None
        if isinstance(details, dict):
            for k in ("ErrorMessage", "FailureReason", "failureReason", "Message", "message", "error"):
                if details.get(k):
                    msg = str(details[k])
                    break
        return SageMakerInvocationError(f"SageMaker invocation {invocation_id} failed: {msg}",
                                        invocation_id=invocation_id, failure_location=location)

    def _wait(self, invocation_id: str, output: str, failure: str | None) -> dict:
        deadline = time.monotonic() + self.timeout
        delay = self.poll_initial
        while True:
            if failure and self._exists(failure):
                raise self._failure(failure, invocation_id)
            if self._exists(output):
                data = json.loads(self._read(output))
                if not isinstance(data, dict):
                    raise ValueError("the SageMaker endpoint returned JSON that is not an object")
                return data
            left = deadline - time.monotonic()
            if left <= 0:
                from synthefy_nori_b200.client import APITimeoutError

                raise APITimeoutError(f"timed out waiting for SageMaker invocation {invocation_id}; the client "
                                      "timeout does not cancel an invocation queued on the endpoint")
            time.sleep(min(delay * (1.0 + 0.25 * random.random()), left))
            delay = min(2.0 * delay, self.poll_max)

    def _cleanup(self, invocation_id: str, locations) -> None:
        for loc in dict.fromkeys(x for x in locations if x):
            bucket, key = parse_s3_uri(loc)
            try:
                self.s3.delete_object(Bucket=bucket, Key=key)
            except Exception as exc:  # noqa: BLE001
                warnings.warn(f"could not delete the staged SageMaker object {loc}: {exc}", RuntimeWarning,
                              stacklevel=3)

    def invoke(self, arrays: dict, metadata: dict, *, model: str) -> dict:
        """Run one staged asynchronous invocation and return the endpoint's JSON result."""
        invocation_id = uuid.uuid4().hex
        key = "/".join(p for p in (self.prefix, self.endpoint_name, invocation_id, "request.tensorfile") if p)
        input_location = f"s3://{self.bucket}/{key}"
        output = failure = None
        pending = False
        fd, path = tempfile.mkstemp(prefix="nori-request-", suffix=".tensorfile")
        os.close(fd)
        try:
            write_tensorfile(path, arrays, {"model": model, **metadata})
            self.s3.upload_file(path, self.bucket, key)
            pending = True  # from here the endpoint may read the input even if this call fails
            resp = self.runtime.invoke_endpoint_async(
                EndpointName=self.endpoint_name, InputLocation=input_location, ContentType=CONTENT_TYPE,
                Accept="application/json", InferenceId=invocation_id, RequestTTLSeconds=REQUEST_TTL_SECONDS,
                InvocationTimeoutSeconds=INVOCATION_TIMEOUT_SECONDS,
                S3OutputPathExtension=f"invocations/{invocation_id}", Filename="result.json")
            if resp.get("InferenceId") not in (None, invocation_id):
                raise RuntimeError(f"InvokeEndpointAsync answered for another InferenceId: {resp.get('InferenceId')!r}")
            output, failure = resp.get("OutputLocation"), resp.get("FailureLocation")
            if not isinstance(output, str) or not output:
                raise RuntimeError("InvokeEndpointAsync returned no OutputLocation")
            for name, loc in (("OutputLocation", output), ("FailureLocation", failure)):
                if loc and not _owned(loc, invocation_id):
                    raise RuntimeError(f"InvokeEndpointAsync returned a {name} outside this invocation's prefix")
            try:
                data = self._wait(invocation_id, output, failure)
            except SageMakerInvocationError:
                pending = False
                raise
            pending = False
        finally:
            os.unlink(path)
            if not pending:
                self._cleanup(invocation_id, [input_location] + [x for x in (output, failure)
                                                                 if _owned(x, invocation_id)])
        if data.get("model") != model:
            raise ValueError(f"SageMaker endpoint model mismatch: requested {model!r}, got {data.get('model')!r}")
        return data
