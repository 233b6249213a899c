"""The training CLI accepts the reference launcher's flag names and maps each onto this
build's settings (CPU: argument parsing and model-config construction only)."""

import json

import pytest

from synthefy_nori_b200.training.cli import _model_config, parse_args


def test_reference_flags_map_onto_settings(tmp_path):
    a = parse_args(["--model", "nori-tiny", "--regression-loss", "pinball", "--regression-quantiles", "0.1,0.5,0.9",
                    "--min-samples", "64", "--max-samples", "512", "--no-qassmax", "--no-target-aware-embedding",
                    "--feature-positional-embedding-type", "learned", "--feature-positional-embedding-num-slots", "64",
                    "--bar-borders-low", "-8", "--bar-borders-high", "8", "--no-prefetch", "--prior", "mixture",
                    "--context-missingness-prob", "0.3", "--heavy-tail-prior-prob", "0.2", "--compile",
                    "--no-mixed-precision", "--task-type", "reg"])
    assert (a.min_rows, a.max_rows, a.prefetch_workers) == (64, 512, 0)
    assert a.augment == {"missing_prob": 0.3, "heavy_prob": 0.2}
    assert any("compile" in n for n in a.notices) and any("bf16" in n for n in a.notices)
    cfg = _model_config(a)
    assert cfg["use_qassmax"] is False and "qass_mode" not in cfg
    assert cfg["use_target_aware_embedding"] is False
    assert cfg["feature_positional_embedding_type"] == "learned"
    assert cfg["feature_positional_embedding_num_slots"] == 64
    dec = cfg["decoder_config"]
    assert dec["regression_quantiles"] == [0.1, 0.5, 0.9] and dec["num_reg_quantiles"] == 3
    assert (dec["bar_borders_low"], dec["bar_borders_high"]) == (-8.0, 8.0)
    # the model builds from that config
    from synthefy_nori_b200.utils.loading import build_model

    m = build_model(dict(cfg))
    assert m.num_reg_quantiles == 3
    # --checkpoint reads an architecture config from JSON
    p = tmp_path / "arch.json"
    p.write_text(json.dumps(cfg))
    b = parse_args(["--checkpoint", str(p), "--regression-loss", "mse"])
    assert b.loss == "mse" and _model_config(b)["feature_positional_embedding_type"] == "learned"


def test_reference_flags_refuse_what_cannot_run():
    with pytest.raises(SystemExit):
        parse_args(["--task-type", "both"])
    with pytest.raises(SystemExit):
        parse_args(["--resume-model-only"])
    a = parse_args(["--resume", "ck.pt", "--resume-model-only"])
    assert a.init_from == "ck.pt" and a.resume is None
