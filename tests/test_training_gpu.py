"""Trainer variants on the native stack: Muon optimizer, point and bar-distribution
losses, loss-spike skip."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(**cfg):
    from synthefy_nori_b200.models.config import preset_config, set_regression_head
    from synthefy_nori_b200.training.prior import PriorConfig, scm_prior_batch
    from synthefy_nori_b200.training.trainer import NoriTrainer, TrainConfig
    from synthefy_nori_b200.utils.loading import build_model

    torch.manual_seed(0)
    mc = preset_config("nori-tiny")
    if cfg.pop("mqa", False):  # shared K/V heads in both sequence attentions
        mc.update(self_share_all_kv_heads=True, cross_share_all_kv_heads=True)
    if cfg.get("loss") in ("mse", "smooth_l1", "huber"):
        set_regression_head(mc, loss=cfg["loss"])
    m = build_model(mc).cuda()
    tr = NoriTrainer(m, TrainConfig(**cfg), torch.device("cuda"))
    b = scm_prior_batch(PriorConfig(max_features=10, pad_features=10), 4, 128, 96, seed=5, device=torch.device("cuda"))
    return tr, b


@pytest.mark.parametrize("cfg", [dict(optimizer="muon", lr=2e-3), dict(loss="mse", lr=1e-3),
                                 dict(loss="huber", lr=1e-3), dict(loss="bar_distribution", lr=1e-3),
                                 dict(lr=1e-3, mqa=True)])
def test_trainer_variants_reduce_loss(cfg):
    tr, b = _setup(ema_decay=0.99, **cfg)
    losses = [tr.train_step(b.x, b.y, b.eval_pos).item() for _ in range(10)]
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < losses[0]


def test_loss_spike_skip_leaves_weights():
    tr, b = _setup(lr=1e-3, loss_spike_factor=2.0, loss_spike_warmup=2)
    for _ in range(3):
        tr.train_step(b.x, b.y, b.eval_pos)
    before = tr.flat.data.clone()
    y = b.y.clone()
    y[:, b.eval_pos:] *= 1e3  # a spike
    tr.train_step(b.x, y, b.eval_pos)
    assert tr.skipped_steps == 1 and torch.equal(before, tr.flat.data)


def test_mask_prediction_training():
    from synthefy_nori_b200.models.config import preset_config
    from synthefy_nori_b200.training.prior import PriorConfig, scm_prior_batch
    from synthefy_nori_b200.training.trainer import NoriTrainer, TrainConfig
    from synthefy_nori_b200.utils.loading import build_model

    cfg = preset_config("nori-tiny")
    cfg["mask_prediction"] = True
    torch.manual_seed(0)
    m = build_model(cfg).cuda()
    assert m.feature_decoder is not None
    tr = NoriTrainer(m, TrainConfig(lr=1e-3, mask_prediction=True), torch.device("cuda"))
    b = scm_prior_batch(PriorConfig(max_features=10, pad_features=10), 4, 128, 96, seed=5, device=torch.device("cuda"))
    losses = [tr.train_step(b.x, b.y, b.eval_pos).item() for _ in range(10)]
    assert all(torch.isfinite(torch.tensor(losses))) and losses[-1] < losses[0]
    assert m.feature_decoder[0].weight.grad is not None and m.feature_decoder[0].weight.grad.abs().sum() > 0


def test_mqa_layouts_follow_the_optimizer():
    """With shared K/V heads the persistent bf16 layouts written after each optimizer step
    equal a fresh cast of the (head-0-broadcast) weights."""
    from synthefy_nori_b200.ops.fused_layer import _bf, _pad_heads, layer_weights

    tr, b = _setup(lr=1e-3, mqa=True)
    for _ in range(2):
        tr.train_step(b.x, b.y, b.eval_pos)
    torch.cuda.synchronize()
    layer = tr.model.transformer_encoder.layers[0]
    persistent = getattr(layer, "_nori_layouts", None)
    assert persistent is not None
    E, H = layer.embed_dim, layer.nhead
    D = E // H
    want = _bf(_pad_heads(layer_weights(layer)["w_ctx"].detach(), H, D, -(-D // 8) * 8))
    torch.testing.assert_close(persistent[1]["w_ctx"].float(), want.float(), atol=0, rtol=0)
