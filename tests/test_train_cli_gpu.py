"""Training CLI: runs, checkpoints atomically, and 2 + 2 resumed steps match 4
uninterrupted steps (to fp32 reduction-order noise: split-K weight gradients and dQ
are summed in L2 in a run-dependent order, and AdamW's normalisation can scale a
difference in a near-zero gradient component up to a few times 1e-5 in the weights)."""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu

ARGS = ["--model", "nori-tiny", "--batch-size", "2", "--min-rows", "64", "--max-rows", "96", "--max-features", "10",
        "--total-steps", "4", "--warmup-steps", "2", "--log-interval", "1", "--save-interval", "2", "--lr", "1e-3"]


def test_resume_matches_uninterrupted(tmp_path):
    from synthefy_nori_b200.training.cli import main
    from synthefy_nori_b200.utils.loading import load_model

    a, b = str(tmp_path / "a"), str(tmp_path / "b")
    assert main(ARGS + ["--checkpoint-dir", a]) == 0
    assert main(ARGS + ["--checkpoint-dir", b, "--run-steps", "2"]) == 0
    ck = torch.load(os.path.join(b, "latest.pt"), map_location="cpu", weights_only=False)
    assert ck["step"] == 2
    assert main(ARGS + ["--checkpoint-dir", b, "--resume", "latest"]) == 0
    sa = torch.load(os.path.join(a, "latest.pt"), map_location="cpu", weights_only=False)
    sb = torch.load(os.path.join(b, "latest.pt"), map_location="cpu", weights_only=False)
    assert sa["step"] == sb["step"] == 4
    for k in sa["model_state_dict"]:
        torch.testing.assert_close(sa["model_state_dict"][k], sb["model_state_dict"][k], atol=2e-4, rtol=1e-3)
    for k in sa["ema_state_dict"]:
        torch.testing.assert_close(sa["ema_state_dict"][k], sb["ema_state_dict"][k], atol=2e-4, rtol=1e-3)
    # the checkpoint loads as a model (EMA weights preferred, like a released checkpoint)
    m = load_model(os.path.join(a, "latest.pt"))
    assert sum(p.numel() for p in m.parameters()) > 0


def test_wcd_schedule_shape():
    from synthefy_nori_b200.training.cli import wcd_lr

    lrs = [wcd_lr(s, 1.0, 10, 50, 100, 0.1) for s in range(100)]
    assert lrs[0] == pytest.approx(0.1) and lrs[9] == pytest.approx(1.0)
    assert all(v == 1.0 for v in lrs[10:50])
    assert lrs[99] == pytest.approx(0.1, abs=1e-3)
    assert all(x >= y for x, y in zip(lrs[50:], lrs[51:]))
