"""The package's top-level names (the reference's public API) and the bundled config files."""

import json

import pytest


def test_top_level_names():
    import synthefy_nori_b200 as nori

    for name in nori.__all__:
        assert getattr(nori, name) is not None, name
    assert nori.NoriRegressor.__name__ == "NoriRegressor"
    assert issubclass(nori.ContextTooLargeError, MemoryError) and issubclass(nori.ContextTooLargeError, RuntimeError)
    with pytest.raises(AttributeError):
        nori.no_such_name  # noqa: B018


def test_bundled_configs_match_definitions():
    from synthefy_nori_b200.configs import (DEFAULT_INFERENCE_CONFIG, DEFAULT_MODEL_CONFIG, MODEL_V3_INFERENCE_CONFIG,
                                            config_path, get_default_inference_config_name)
    from synthefy_nori_b200.inference import preprocess
    from synthefy_nori_b200.models.config import base_config

    def load(name):
        with open(config_path(name)) as f:
            return json.load(f)

    assert load(DEFAULT_INFERENCE_CONFIG) == json.loads(json.dumps(preprocess.DEFAULT_INFERENCE_CONFIG))
    assert load(MODEL_V3_INFERENCE_CONFIG) == json.loads(json.dumps(preprocess.MODEL_V3_INFERENCE_CONFIG))
    assert load(DEFAULT_MODEL_CONFIG) == json.loads(json.dumps(base_config()))
    assert get_default_inference_config_name("nori-1-5") == MODEL_V3_INFERENCE_CONFIG
    assert get_default_inference_config_name("nori-6m") == DEFAULT_INFERENCE_CONFIG
    # a config given by bundled name or by path resolves to its members
    by_name = preprocess.resolve_inference_config(MODEL_V3_INFERENCE_CONFIG)
    by_path = preprocess.resolve_inference_config(config_path(MODEL_V3_INFERENCE_CONFIG))
    assert by_name == by_path == json.loads(json.dumps(preprocess.MODEL_V3_INFERENCE_CONFIG))


def test_context_too_large_when_subsampling_is_forbidden():
    from synthefy_nori_b200.inference.memory_policy import ContextTooLargeError, MemoryPolicy

    pol = MemoryPolicy(allow_subsample=False, offload_to_host=False)
    with pytest.raises(ContextTooLargeError, match="allow_subsample"):
        pol.resolve(n_context_rows=10_000_000, n_groups=250, nlayers=26, embed_dim=448, head_dim=56,
                    device_total_gb=1.0)
    with pytest.raises(MemoryError):  # the memory ladder's handlers still catch it
        pol.resolve(n_context_rows=10_000_000, n_groups=250, nlayers=26, embed_dim=448, head_dim=56,
                    device_total_gb=1.0)
