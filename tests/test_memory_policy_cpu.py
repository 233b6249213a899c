"""MemoryPolicy coercion, validation and rung resolution; client local mode."""

import numpy as np
import pytest

from synthefy_nori_b200.inference.memory_policy import MemoryPolicy, estimate_cache_gb, int8_footprint_gb


def test_presets_and_coercion():
    assert MemoryPolicy.coerce(None) == MemoryPolicy()
    assert MemoryPolicy.coerce("exact").allow_quantization is False
    assert MemoryPolicy.coerce("max_context").cache_dtype == "int8"
    assert MemoryPolicy.coerce("off").cache is False
    assert MemoryPolicy.coerce({"gpu_budget_frac": 0.25}).gpu_budget_frac == 0.25
    with pytest.raises(ValueError):
        MemoryPolicy.coerce("fastest")
    with pytest.raises(Exception):
        MemoryPolicy(unknown_field=1)
    with pytest.raises(TypeError):
        MemoryPolicy.coerce(3)


def test_cache_size_formula():
    gb = estimate_cache_gb(n_context_rows=100_000, n_groups=51, nlayers=26, embed_dim=448)
    assert abs(gb - 26 * 51 * 100_000 * 2 * 448 * 2 / 1024 ** 3) < 1e-9
    assert abs(int8_footprint_gb(gb, head_dim=56) - gb / 2 * (1 + 4 / 56)) < 1e-9


@pytest.mark.parametrize("rows,total,gpus,rung", [(1000, 180, 1, "resident_bf16"), (100_000, 180, 1, "resident_int8"),
                                                  (400_000, 180, 8, "context_sharded_int8"),
                                                  (400_000, 180, 1, "subsample")])
def test_resolve_rungs(rows, total, gpus, rung):
    # 100k rows of nori-100m: 221 GiB bf16, 119 GiB int8 -> resident int8 within an 80% budget
    p = MemoryPolicy(gpu_budget_frac=0.8).resolve(n_context_rows=rows, n_groups=51, nlayers=26, embed_dim=448, head_dim=56,
                               device_total_gb=total, n_gpus=gpus)
    assert p.rung == rung
    if rung == "subsample":
        assert 0 < p.dropped_context_rows < rows


def test_exact_never_quantizes_and_off_has_no_cache():
    p = MemoryPolicy.coerce("exact").resolve(n_context_rows=100_000, n_groups=51, nlayers=26, embed_dim=448,
                                             head_dim=56, device_total_gb=180)
    assert p.rung == "subsample"
    assert MemoryPolicy.coerce("off").resolve(n_context_rows=10, n_groups=3, nlayers=2, embed_dim=64, head_dim=32,
                                              device_total_gb=10).rung == "no_cache"


def test_client_local_mode_and_multi_target():
    from synthefy_nori_b200.client import SynthefyNoriClient

    rng = np.random.default_rng(0)
    X = rng.standard_normal((60, 4)).astype(np.float32)
    Y = np.stack([X @ rng.standard_normal(4), X[:, 0] ** 2], -1)
    c = SynthefyNoriClient(mode="local", model="nori-tiny", weights="random", device="cpu")
    out = c.predict(X[:50], Y[:50], X[50:])
    assert out.shape == (10, 2)
    with pytest.raises(ValueError):
        SynthefyNoriClient(mode="remote")  # no model named
    with pytest.raises(ValueError):
        SynthefyNoriClient(mode="remote", model="nori-6m", api_key="")  # no key
