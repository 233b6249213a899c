"""CUDA-graph replay of the cached query pass (``GraphedQueryRunner``) against the eager
cached pass: same outputs for bf16 and int8 caches, query counts that are not a multiple
of the captured chunk (padded last chunk), and repeated replays."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cache_dtype", ["bf16", "int8"])
def test_graphed_query_runner_matches_eager(cache_dtype):
    from synthefy_nori_b200.inference.cuda_graphs import GraphedQueryRunner
    from synthefy_nori_b200.models.config import preset_config
    from synthefy_nori_b200.utils.loading import build_model

    torch.manual_seed(0)
    dev = torch.device("cuda")
    model = build_model(preset_config("nori-tiny")).to(dev).eval()
    B, n_ctx, F = 2, 200, 7
    x = torch.randn(B, n_ctx + 300, F, device=dev)
    y = x[..., 0] * 0.5 + torch.sin(x[..., 1])
    with torch.no_grad():
        cache = model.build_context_cache(x[:, :n_ctx], y[:, :n_ctx], cache_dtype=cache_dtype)
        xq = x[:, n_ctx:]
        eager = model.apply_context_cache(xq, cache).float()
    runner = GraphedQueryRunner(model, cache, B, 128, F, dev)
    for _ in range(2):  # replays are repeatable
        got = runner(xq).float()
        assert got.shape == eager.shape
        torch.testing.assert_close(got, eager, atol=2e-2, rtol=2e-2)
    # a short call (one padded chunk)
    got = runner(xq[:, :37]).float()
    torch.testing.assert_close(got, eager[:, :37], atol=2e-2, rtol=2e-2)
