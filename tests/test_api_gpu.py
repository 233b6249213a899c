"""NoriRegressor on the native CUDA path vs the CPU (PyTorch) path, and the native
quantile decode vs its PyTorch statement."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_quantile_decode_kernel_matches_torch():
    from synthefy_nori_b200 import ops
    from synthefy_nori_b200.inference.predictor import decode_torch

    torch.manual_seed(0)
    taus = torch.tensor([(i + 1) / 1000 for i in range(999)], device="cuda")
    raw = torch.randn(33, 999, device="cuda")
    lv = torch.tensor([0.0005, 0.1, 0.5, 0.9, 0.9995], device="cuda")
    m, q, s = ops.quantile_decode(raw, taus, lv, True)
    rm, rq, rs = decode_torch(raw, taus, lv, True)
    torch.testing.assert_close(s, rs)
    torch.testing.assert_close(m, rm, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(q, rq, atol=1e-5, rtol=1e-5)


def test_regressor_cuda_matches_cpu():
    from synthefy_nori_b200.api import NoriRegressor

    rng = np.random.default_rng(0)
    X = rng.standard_normal((140, 6)).astype(np.float32)
    y = X @ rng.standard_normal(6) + 0.1 * rng.standard_normal(140)
    kw = dict(model="nori-tiny", weights="random", n_estimators=2)
    cpu = NoriRegressor(device="cpu", **kw).fit(X[:100], y[:100])
    gpu = NoriRegressor(device="cuda", **kw).fit(X[:100], y[:100])
    a, b = cpu.predict(X[100:]), gpu.predict(X[100:])
    assert np.max(np.abs(a - b)) < 0.05 * np.std(y) + 1e-3
    qa = cpu.predict(X[100:], output_type="quantiles", quantiles=[0.1, 0.9])
    qb = gpu.predict(X[100:], output_type="quantiles", quantiles=[0.1, 0.9])
    assert np.max(np.abs(qa - qb)) < 0.08 * np.std(y) + 1e-3


def test_default_ensemble_cuda_matches_cpu():
    """Eight reference-config members (quantile / adaptive rebalancing, SVD features,
    fingerprint, shuffles) preprocessed on the device, batched by width."""
    from synthefy_nori_b200.api import NoriRegressor

    rng = np.random.default_rng(1)
    X = rng.standard_normal((300, 9)).astype(np.float32)
    X[:, 2] = np.exp(X[:, 2])
    X[rng.random(X.shape) < 0.05] = np.nan
    y = np.nan_to_num(X) @ rng.standard_normal(9) + 0.1 * rng.standard_normal(300)
    kw = dict(model="nori-tiny", weights="random")
    cpu = NoriRegressor(device="cpu", **kw).fit(X[:240], y[:240])
    gpu = NoriRegressor(device="cuda", **kw).fit(X[:240], y[:240])
    a, b = cpu.predict(X[240:]), gpu.predict(X[240:])
    assert gpu.predictor_.n_estimators == 8
    assert np.max(np.abs(a - b)) < 0.05 * np.std(y) + 1e-3
    e = gpu.get_embeddings(X[240:])
    assert e.shape[:2] == (8, 60) and np.all(np.isfinite(e))


def test_cuda_graph_replay_matches_eager():
    from synthefy_nori_b200.inference.predictor import NoriPredictor
    from synthefy_nori_b200.models.config import preset_config
    from synthefy_nori_b200.utils.loading import build_model

    torch.manual_seed(0)
    model = build_model(preset_config("nori-6m")).cuda().eval()
    rng = np.random.default_rng(2)
    X = rng.standard_normal((900, 12)).astype(np.float32)
    y = X[:, 0] - X[:, 1] ** 2
    eager = NoriPredictor(model, "cuda", n_estimators=2)
    graphed = NoriPredictor(model, "cuda", n_estimators=2, cuda_graphs=True, graph_rows=128)
    ce, cg = eager.fit_context(X[:600], y[:600]), graphed.fit_context(X[:600], y[:600])
    a = eager.predict_raw(ce, X[600:])
    b = graphed.predict_raw(cg, X[600:])  # 300 rows: two full chunks and a padded one
    torch.testing.assert_close(b, a, atol=2e-3, rtol=2e-3)
    b2 = graphed.predict_raw(cg, X[600:700])  # replay
    torch.testing.assert_close(b2, a[:100], atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("placement,rows", [("offload", None), ("stream", 64), ("stream", 37)])
@pytest.mark.parametrize("dtype", ["bf16", "int8"])
def test_host_offloaded_and_streamed_caches_match_resident(placement, rows, dtype):
    """Host-offloaded caches (a layer copied in just before it runs) and streamed caches
    (row blocks merged by their log-sum-exps) give the resident cache's predictions."""
    from synthefy_nori_b200.models.config import preset_config
    from synthefy_nori_b200.utils.loading import build_model

    torch.manual_seed(0)
    dev = torch.device("cuda")
    model = build_model(preset_config("nori-tiny")).to(dev).eval()
    x = torch.randn(2, 300, 6, device=dev)
    y = x[..., 0] - 0.5 * x[..., 1] ** 2
    with torch.no_grad():
        ref = model.apply_context_cache(x[:, 200:], model.build_context_cache(x[:, :200], y[:, :200],
                                                                              cache_dtype=dtype)).float()
        c = model.build_context_cache(x[:, :200], y[:, :200], cache_dtype=dtype, placement=placement,
                                      stream_block_rows=rows)
        got = model.apply_context_cache(x[:, 200:], c).float()
    torch.testing.assert_close(got, ref, atol=3e-2, rtol=3e-2)
