"""Native two-phase encoder (Model v3 / nori-1-5) inference against the PyTorch module in
fp32 on the same GPU, and the per-head query/key norm kernel against its fp32 formula."""

import math

import pytest
import torch

from synthefy_nori_b200.models.config import preset_config
from synthefy_nori_b200.utils.loading import build_model

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12))


def test_head_rmsnorm_matches_formula():
    from synthefy_nori_b200 import ops

    torch.manual_seed(0)
    for H, D, rows, ld in ((2, 32, 77, 128), (8, 56, 300, 448), (4, 64, 5, 264)):
        x = torch.randn(rows, ld, device="cuda").to(torch.bfloat16)
        gain = torch.rand(D, device="cuda") + 0.5
        ref = x.float().clone()
        blk = ref[:, : H * D].view(rows, H, D)
        blk = blk * torch.rsqrt(blk.pow(2).mean(-1, keepdim=True) + 1e-6) * gain * 2.5
        ref[:, : H * D] = blk.reshape(rows, H * D)
        ops.head_rmsnorm_(x, H, D, gain, 1e-6, 2.5)
        torch.testing.assert_close(x.float(), ref, atol=2e-2, rtol=1e-2)
        # columns past the heads are untouched
        assert torch.equal(x[:, H * D:].float(), ref[:, H * D:].to(torch.bfloat16).float())


def _model(tp, seed=0):
    cfg = preset_config("nori-tiny")
    cfg["two_phase_config"] = dict(tp)
    torch.manual_seed(seed)
    return build_model(cfg).cuda().eval()


@pytest.mark.parametrize("B,R,G,eval_pos", [(1, 60, 3, 40), (2, 300, 5, 201)])
def test_native_two_phase_encoder_matches_module(B, R, G, eval_pos):
    from synthefy_nori_b200.ops import two_phase as native_two_phase

    model = _model({"target_tokens": 2, "row_layers": 2, "row_heads": 2, "row_hidden_dim": 96})
    enc = model.transformer_encoder
    assert native_two_phase.supported(enc)
    g = torch.Generator(device="cuda").manual_seed(1)
    cells = torch.randn(B, R, G, enc.cell_dim, device="cuda", generator=g)
    y = torch.randn(B, R, device="cuda", generator=g)
    y[:, eval_pos:] = float("nan")
    with torch.no_grad():
        rows_ref, cells_ref = enc(cells, y, eval_pos)
        rows, cell_states = native_two_phase.forward(enc, cells, y, eval_pos)
    torch.cuda.synchronize()
    assert rows.dtype == torch.bfloat16 and rows.shape == rows_ref.shape
    assert _rel(rows, rows_ref) < 3e-2, _rel(rows, rows_ref)
    assert _rel(cell_states, cells_ref) < 3e-2, _rel(cell_states, cells_ref)


def test_model_forward_uses_native_two_phase():
    model = _model({"target_tokens": 2, "row_layers": 1, "row_heads": 2, "row_hidden_dim": 96})
    torch.manual_seed(4)
    x = torch.randn(1, 90, 6, device="cuda")
    y = torch.randn(1, 60, device="cuda")
    with torch.no_grad():
        assert model.use_native_two_phase(x.device)
        out = model(x, y, 60, task_type="reg")
        model.impl = "torch"
        ref = model(x, y, 60, task_type="reg")
        model.impl = "auto"
    assert out.shape == ref.shape
    assert _rel(out, ref) < 3e-2, _rel(out, ref)
    # with autograd on the module runs (the native path is inference-only)
    assert not model.use_native_two_phase(x.device) or not torch.is_grad_enabled()


def test_log_factor_matches_module_scaling():
    from synthefy_nori_b200.ops.two_phase import _log_factor

    assert _log_factor(1) == 1.0
    assert math.isclose(_log_factor(2), math.log(2.0))
    assert math.isclose(_log_factor(1000), math.log(1000.0))
