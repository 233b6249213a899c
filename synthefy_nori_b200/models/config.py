"""Architecture records (``model_config`` dicts) and named presets.

A ``model_config`` dict is the architecture record stored in every Nori checkpoint
(reference ``src/synthefy_nori/configs/model_base.json`` plus the overrides that the
training CLI applies, ``training/cli.py:1249-1326``).  The same keys are used here so
that checkpoints written by either implementation load in the other.

Presets:

* ``nori-6m``: the shipped recipe - 16 layers, E=128, hid 384, 2 heads, "v2-lite"
  (SwiGLU, RMSNorm, pre-norm, DeepNorm alpha = L**-0.5, RBF cells), QASS ``full``,
  target-aware + column-specific y embedding, 999 pinball quantiles (reference
  ``scripts/train.sh:117-157``).  5.82M parameters.
* ``nori-30m`` / ``nori-100m``: the released checkpoints' dimensions are not published
  in the reference tree (only parameter counts, 29.2M / 98.3M, and head widths 44 / 56
  mentioned in ``model/layer.py:860``).  Random-init configs with those head widths
  and parameter counts within 1% are chosen here; a downloaded checkpoint always
  carries its own ``model_config``, which takes precedence.
"""

from __future__ import annotations

import copy
import os

QUANTILES_999 = [round((i + 1) / 1000.0, 4) for i in range(999)]

BASE_CONFIG = {
    "preprocess_config_x": {
        "num_features": 2,
        "nan_handling_enabled": True,
        "normalize_on_train_only": True,
        "normalize_x": True,
        "remove_outliers": False,
        "normalize_by_used_features": True,
    },
    "encoder_config_x": {
        "num_features": 2,
        "embedding_size": 96,
        "mask_embedding_size": 96,
        "encoder_use_bias": True,
        "numeric_embed_type": "RBF",
        "RBF_config": {
            "token_embed_dim": 16,
            "n_kernels": 64,
            "sigma": 0.5,
            "use_learn_sigma": False,
            "use_learn_embeddings": False,
            "use_original_features": False,
        },
    },
    "encoder_config_y": {"num_inputs": 1, "embedding_size": 96, "nan_handling_y_encoder": True, "max_num_classes": 10},
    "decoder_config": {"num_classes": 10},
    "feature_positional_embedding_type": "none",
    "nlayers": 12,
    "nhead": 6,
    "embed_dim": 96,
    "hid_dim": 384,
    "features_per_group": 2,
    "dropout": 0,
    "pre_norm": False,
    "activation": "gelu",
    "recompute_attn": False,
    "layer_arch": "smf",
    "self_share_all_kv_heads": False,
    "cross_share_all_kv_heads": False,
    "seq_attn_isolated": True,
    "seq_attn_serial": False,
    "mask_prediction": False,
}

ATTENTION_SCALE_DEFAULTS = {"use_logn_attention": False, "use_learnable_attn_temperature": False, "attn_n_ref": 1024.0}


def base_config() -> dict:
    return copy.deepcopy(BASE_CONFIG)


def set_dims(cfg: dict, *, embed_dim=None, hid_dim=None, nhead=None, nlayers=None) -> dict:
    if embed_dim is not None:
        cfg["embed_dim"] = embed_dim
        for sub in ("encoder_config_x", "encoder_config_y"):
            for f in ("embedding_size", "mask_embedding_size"):
                if f in cfg[sub]:
                    cfg[sub][f] = embed_dim
    if hid_dim is not None:
        cfg["hid_dim"] = hid_dim
    if nhead is not None:
        cfg["nhead"] = nhead
    if nlayers is not None:
        cfg["nlayers"] = nlayers
    return cfg


def apply_v2_lite(cfg: dict) -> dict:
    cfg["activation"] = "swiglu"
    cfg["norm_type"] = "rmsnorm"
    cfg["pre_norm"] = True
    cfg["deepnorm_alpha"] = cfg["nlayers"] ** (-0.5)
    return cfg


def set_regression_head(cfg: dict, quantiles=None, loss: str = "pinball") -> dict:
    dec = cfg.setdefault("decoder_config", {})
    dec["regression_loss"] = loss
    if loss == "pinball":
        qs = list(quantiles if quantiles is not None else QUANTILES_999)
        dec["num_reg_quantiles"] = len(qs)
        dec["regression_quantiles"] = [float(q) for q in qs]
    elif loss in ("mse", "smooth_l1", "huber"):  # one point prediction per row
        dec["num_reg_quantiles"] = 1
        dec.pop("regression_quantiles", None)
    return cfg


def finalize_arch_config(cfg: dict) -> dict:
    """Pin every architecture flag that ``build_model`` would otherwise default
    (QASS mode; attention-scale flags).  ``SYNTHEFY_QASS_MODE`` may override the QASS
    mode here and only here (reference ``utils/loading.py:62-99``)."""
    if bool(cfg.get("use_qassmax", False)):
        env = os.environ.get("SYNTHEFY_QASS_MODE")
        cfg["qass_mode"] = env.strip().lower() if env else str(cfg.get("qass_mode") or "full")
    for k, v in ATTENTION_SCALE_DEFAULTS.items():
        cfg.setdefault(k, v)
    return cfg


def _preset(embed_dim, hid_dim, nhead, nlayers, quantiles=None) -> dict:
    cfg = set_dims(base_config(), embed_dim=embed_dim, hid_dim=hid_dim, nhead=nhead, nlayers=nlayers)
    apply_v2_lite(cfg)
    cfg["use_qassmax"] = True
    cfg["use_target_aware_embedding"] = True
    cfg["use_column_specific_y_aware"] = True
    cfg["omit_feature_decoder"] = False
    set_regression_head(cfg, quantiles)
    return finalize_arch_config(cfg)


PRESETS = {
    "nori-6m": dict(embed_dim=128, hid_dim=384, nhead=2, nlayers=16),
    # head width 44: 8 heads x 44 = 352
    "nori-30m": dict(embed_dim=352, hid_dim=1056, nhead=8, nlayers=12),
    # head width 56: 8 heads x 56 = 448
    "nori-100m": dict(embed_dim=448, hid_dim=1344, nhead=8, nlayers=26),
    # small config for tests and smoke runs
    "nori-tiny": dict(embed_dim=64, hid_dim=96, nhead=2, nlayers=2),
}


def preset_config(name: str, quantiles=None) -> dict:
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; choose one of {sorted(PRESETS)}")
    return _preset(quantiles=quantiles, **PRESETS[name])
