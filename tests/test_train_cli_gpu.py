"""Training CLI: runs, checkpoints atomically, and 2 + 2 resumed steps match 4
uninterrupted steps (to fp32 reduction-order noise: split-K weight gradients and dQ
are summed in L2 in a run-dependent order, and AdamW's normalisation can turn a
difference in a near-zero gradient component into a full-size update of that element,
so the check compares whole updates, not single elements)."""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu

ARGS = ["--model", "nori-tiny", "--batch-size", "2", "--min-rows", "64", "--max-rows", "96", "--max-features", "10",
        "--total-steps", "4", "--warmup-steps", "2", "--log-interval", "1", "--save-interval", "2", "--lr", "1e-3"]


def _delta_ratio(end_a, end_b, start):
    """||(a - s) - (b - s)|| / ||a - s|| over every floating tensor of a state dict."""
    num = den = 0.0
    for k, s0 in start.items():
        if not torch.is_floating_point(s0):
            continue
        da = end_a[k].double() - s0.double()
        db = end_b[k].double() - s0.double()
        num += float((da - db).pow(2).sum())
        den += float(da.pow(2).sum())
    return (num / max(den, 1e-30)) ** 0.5


def test_resume_matches_uninterrupted(tmp_path):
    """The two resumed steps move the weights (and the EMA) the same way as steps 3-4 of
    the uninterrupted run, up to fp32 reduction-order noise. A resume that lost the AdamW
    moments, the step count, the LR schedule or the EMA would change that update by a large
    fraction of its size; reduction-order noise changes it by well under one percent."""
    import shutil

    from synthefy_nori_b200.training.cli import main
    from synthefy_nori_b200.utils.loading import load_model

    a, b = str(tmp_path / "a"), str(tmp_path / "b")
    assert main(ARGS + ["--checkpoint-dir", a]) == 0
    assert main(ARGS + ["--checkpoint-dir", b, "--run-steps", "2"]) == 0
    ck = torch.load(os.path.join(b, "latest.pt"), map_location="cpu", weights_only=False)
    assert ck["step"] == 2
    shutil.copy(os.path.join(b, "latest.pt"), str(tmp_path / "step2.pt"))
    assert main(ARGS + ["--checkpoint-dir", b, "--resume", "latest"]) == 0
    sa = torch.load(os.path.join(a, "latest.pt"), map_location="cpu", weights_only=False)
    sb = torch.load(os.path.join(b, "latest.pt"), map_location="cpu", weights_only=False)
    assert sa["step"] == sb["step"] == 4
    assert _delta_ratio(sa["model_state_dict"], sb["model_state_dict"], ck["model_state_dict"]) < 0.05
    assert _delta_ratio(sa["ema_state_dict"], sb["ema_state_dict"], ck["ema_state_dict"]) < 0.05
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
