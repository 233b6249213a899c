"""Client remote mode against the framework's own HTTP server (uvicorn on 127.0.0.1),
retry behaviour against a server that fails first."""

import socket
import threading
import time

import numpy as np
import pytest


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.fixture(scope="module")
def server():
    import uvicorn

    from synthefy_nori_b200.serving import create_app

    port = _free_port()
    cfg = uvicorn.Config(create_app(default_model="nori-tiny", weights="random", device="cpu", api_key="k"),
                         host="127.0.0.1", port=port, log_level="error")
    srv = uvicorn.Server(cfg)
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    for _ in range(200):
        if srv.started:
            break
        time.sleep(0.05)
    yield f"http://127.0.0.1:{port}"
    srv.should_exit = True
    th.join(timeout=10)


def _data():
    rng = np.random.default_rng(0)
    X = rng.standard_normal((70, 4)).astype(np.float32)
    X[3, 1] = np.nan
    y = X[:, 0] * 2 + 0.1 * rng.standard_normal(70)
    return X[:50], y[:50], X[50:]


def test_remote_matches_local(server):
    from synthefy_nori_b200.client import APIError, SynthefyNoriClient

    Xtr, ytr, Xte = _data()
    local = SynthefyNoriClient(mode="local", model="nori-tiny", weights="random", device="cpu")
    with SynthefyNoriClient("k", mode="remote", model="nori-tiny", base_url=server) as remote:
        np.testing.assert_allclose(remote.predict(Xtr, ytr, Xte), local.predict(Xtr, ytr, Xte), rtol=1e-5, atol=1e-5)
        q = remote.predict(Xtr, ytr, Xte, output_type="quantiles", quantiles=[0.1, 0.9])
        assert q.shape == (2, 20)
        full = remote.predict(Xtr, ytr, Xte, output_type="full")
        assert full["quantiles"].shape[0] == 20
        with pytest.raises(ValueError):
            remote.predict(Xtr, np.r_[ytr[:-1], np.nan], Xte)
    with SynthefyNoriClient("wrong", mode="remote", model="nori-tiny", base_url=server, max_retries=0) as bad:
        with pytest.raises(APIError) as e:
            bad.predict(Xtr, ytr, Xte)
        assert e.value.status_code == 401


def test_retries_on_503():
    import httpx

    from synthefy_nori_b200.client import SynthefyNoriClient

    calls = {"n": 0}

    def handler(request):
        calls["n"] += 1
        if calls["n"] < 3:
            return httpx.Response(503, headers={"retry-after": "0"})
        return httpx.Response(200, json={"task": "regression", "predictions": [1.0, None]})

    c = SynthefyNoriClient("k", mode="remote", model="nori-6m", base_url="http://x", max_retries=2)
    c.http = httpx.Client(base_url="http://x", transport=httpx.MockTransport(handler))
    out = c.predict(np.zeros((3, 2)), np.zeros(3), np.zeros((2, 2)))
    assert calls["n"] == 3 and out[0] == 1.0 and np.isnan(out[1])
