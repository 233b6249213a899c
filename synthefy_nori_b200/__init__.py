"""Nori on Blackwell: a B200-native tabular foundation model framework.

The top-level names are the reference package's public API (``synthefy_nori/__init__.py``);
they are imported on first use, so ``import synthefy_nori_b200`` stays light.
"""

from __future__ import annotations

import importlib

__version__ = "0.1.0"

_EXPORTS = {
    "NoriRegressor": "api", "infer": "api", "predict": "api",
    "NoriEmbedding": "embedding",
    "billable_price": "pricing",
    "MemoryPolicy": "inference.memory_policy", "ContextTooLargeError": "inference.memory_policy",
    "ContextSubsampledWarning": "inference.degradation", "DegradedPipelineWarning": "inference.degradation",
    "SvdFallbackWarning": "inference.degradation", "strict_pipeline": "inference.degradation",
    "DEFAULT_MULTI_TARGET_PREDICTION_STRATEGY": "multi_target", "MultiTargetPredictionPolicy": "multi_target",
    "DEFAULT_INFERENCE_CONFIG": "configs", "DEFAULT_MODEL_CONFIG": "configs", "MODEL_V3_INFERENCE_CONFIG": "configs",
    "config_path": "configs",
}
__all__ = sorted(_EXPORTS) + ["discretize"]


def __getattr__(name: str):
    if name == "discretize":
        return importlib.import_module("synthefy_nori_b200.discretize")
    if name in _EXPORTS:
        value = getattr(importlib.import_module(f"synthefy_nori_b200.{_EXPORTS[name]}"), name)
        globals()[name] = value
        return value
    raise AttributeError(f"module 'synthefy_nori_b200' has no attribute {name!r}")
