"""Bundled configuration files and their names.

* ``default_inference.json``: the preprocessing ensemble (eight members) of every model
  without an entry in :data:`INFERENCE_CONFIG_BY_MODEL_NAME` (the released nori-6m / 30m /
  100m weights, and checkpoints loaded by path);
* ``model_v3_inference.json``: the four-member ensemble of ``nori-1-5``;
* ``model_base.json``: the training / architecture base config (encoders, embedding sizes,
  RBF kernels) that the presets and the training CLI start from.

The files are the JSON form of ``inference.preprocess.DEFAULT_INFERENCE_CONFIG`` /
``MODEL_V3_INFERENCE_CONFIG`` and ``models.config.base_config()`` (a test keeps them equal),
in the reference's schema (``src/synthefy_nori/configs``), so configs written for either
load in both.
"""

from __future__ import annotations

import json
import os

DEFAULT_INFERENCE_CONFIG = "default_inference.json"
MODEL_V3_INFERENCE_CONFIG = "model_v3_inference.json"
DEFAULT_MODEL_CONFIG = "model_base.json"
INFERENCE_CONFIG_BY_MODEL_NAME = {"nori-1-5": MODEL_V3_INFERENCE_CONFIG}

_HERE = os.path.dirname(os.path.abspath(__file__))


def config_path(filename: str = DEFAULT_INFERENCE_CONFIG) -> str:
    """Absolute path of a bundled config file."""
    return os.path.join(_HERE, filename)


def get_default_inference_config_name(model_name: str | None) -> str:
    """The bundled inference config a released model uses when the caller passes none."""
    return INFERENCE_CONFIG_BY_MODEL_NAME.get(model_name or "", DEFAULT_INFERENCE_CONFIG)


def load_config(name_or_path: str):
    """A bundled config by file name, or any JSON config file by path."""
    path = name_or_path if os.path.isfile(name_or_path) else config_path(name_or_path)
    with open(path) as f:
        return json.load(f)


__all__ = ["DEFAULT_INFERENCE_CONFIG", "MODEL_V3_INFERENCE_CONFIG", "DEFAULT_MODEL_CONFIG",
           "INFERENCE_CONFIG_BY_MODEL_NAME", "config_path", "get_default_inference_config_name", "load_config"]
