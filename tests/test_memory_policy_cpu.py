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


@pytest.mark.parametrize("rows,total,gpus,host,rung", [(1000, 180, 1, 0, "resident_bf16"),
                                                       (100_000, 180, 1, 0, "resident_int8"),
                                                       (400_000, 180, 8, 0, "context_sharded_int8"),
                                                       (400_000, 180, 1, 0, "subsample"),
                                                       (400_000, 180, 1, 2000, "offload_bf16"),
                                                       (400_000, 180, 8, 2000, "context_sharded_int8"),
                                                       (400_000, 180, 1, 1000, "offload_int8")])
def test_resolve_rungs(rows, total, gpus, host, rung):
    # 100k rows of nori-100m: 221 GiB bf16, 119 GiB int8 -> resident int8 within an 80% budget;
    # 400k rows: 884 GiB bf16 / 474 GiB int8 -> host offload when the host budget allows it
    p = MemoryPolicy(gpu_budget_frac=0.8).resolve(n_context_rows=rows, n_groups=51, nlayers=26, embed_dim=448,
                                                  head_dim=56, device_total_gb=total, n_gpus=gpus,
                                                  host_total_gb=host)
    assert p.rung == rung
    if rung == "subsample":
        assert 0 < p.dropped_context_rows < rows


def test_exact_never_quantizes_and_off_has_no_cache():
    p = MemoryPolicy.coerce("exact").resolve(n_context_rows=100_000, n_groups=51, nlayers=26, embed_dim=448,
                                             head_dim=56, device_total_gb=180, host_total_gb=0)
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


def test_stream_rung_escalation_and_host_memory(tmp_path):
    from synthefy_nori_b200.inference.memory_policy import host_memory_gb

    p = MemoryPolicy(stream_context=True).resolve(n_context_rows=100_000, n_groups=51, nlayers=26, embed_dim=448,
                                                  head_dim=56, device_total_gb=180, host_total_gb=1000)
    assert p.rung == "stream_bf16" and p.context_row_chunk == 16384 and p.reuse_context_cache is False
    assert p.placement() == ("bf16", "stream", 16384)
    with pytest.raises(ValueError):
        MemoryPolicy(stream_context=True, offload_to_host=False).resolve(
            n_context_rows=10, n_groups=3, nlayers=2, embed_dim=64, head_dim=32, device_total_gb=10)
    r = MemoryPolicy(gpu_budget_frac=0.8).resolve(n_context_rows=1000, n_groups=51, nlayers=26, embed_dim=448,
                                                  head_dim=56, device_total_gb=180)
    chain = [r.rung]
    while (nxt := r.next_rung()) is not None:
        r = r.escalated(nxt)
        chain.append(r.rung)
    assert chain == ["resident_bf16", "resident_int8", "offload_int8", "stream_int8"]
    assert r.placement()[1] == "stream"
    # host memory: the smaller of MemAvailable and the cgroup limit
    mi = tmp_path / "meminfo"
    mi.write_text("MemTotal: 100000000 kB\nMemAvailable: 52428800 kB\n")
    cg = tmp_path / "memory.max"
    cg.write_text(str(20 * 1024 ** 3))
    assert abs(host_memory_gb(str(mi), (str(cg),)) - 20.0) < 1e-9
    cg.write_text("max")
    assert abs(host_memory_gb(str(mi), (str(cg),)) - 50.0) < 1e-9
