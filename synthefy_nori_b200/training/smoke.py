"""One tiny native forward + backward + optimizer step (driver smoke test)."""

from __future__ import annotations

import torch


def run_smoke(device: torch.device) -> float:
    from synthefy_nori_b200 import ops
    from synthefy_nori_b200.models.config import preset_config
    from synthefy_nori_b200.training.prior import PriorConfig, scm_prior_batch
    from synthefy_nori_b200.training.trainer import NoriTrainer, TrainConfig
    from synthefy_nori_b200.utils.loading import build_model

    if not ops.native_available():
        raise RuntimeError(f"native extension not loaded: {ops.native_import_error()}")
    torch.manual_seed(0)
    model = build_model(preset_config("nori-tiny"))
    trainer = NoriTrainer(model, TrainConfig(), device)
    batch = scm_prior_batch(PriorConfig(max_features=12, pad_features=12), 2, 96, 64, seed=1, device=device)
    loss = trainer.train_step(batch.x, batch.y, batch.eval_pos)
    val = float(loss.item())
    ops.check_status(device)
    if not torch.isfinite(torch.tensor(val)):
        raise RuntimeError(f"smoke loss is not finite: {val}")
    print(f"smoke ok: loss={val:.5f}")
    return val
