"""The tensor-core QASS kernels (tcgen05, two tile slots, gradient sums as MMAs) against
the fp32 PyTorch statement and against the mma.sync kernels, over shapes with partial
tiles, several tiles per CTA (both slots in use), padded head widths and 2..8 heads."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from synthefy_nori_b200.models.layers import QASSMaxScaling  # noqa: E402
from synthefy_nori_b200.ops.fused_layer import Geometry, _qass_apply, _qass_apply_torch, _qass_backward, _qass_params  # noqa: E402


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-30))


def _run(params, q, H, D, dq_out, n_keys=777):
    out = _qass_apply(params, "full", q, n_keys, H, D)
    g = Geometry(B=1, ep=n_keys, nq=0, T=1, E=H * D, H=H)
    dq, grads = _qass_backward(params, "full", q, n_keys, g, dq_out)
    return out, dq, grads


@pytest.mark.parametrize("H,D", [(8, 56), (2, 64), (8, 48), (4, 32)])
@pytest.mark.parametrize("R", [333, 40000])
def test_qass_tc_matches_reference_and_legacy(H, D, R, monkeypatch):
    torch.manual_seed(H * 100 + D)
    mod = QASSMaxScaling(num_heads=H, head_dim=D, hidden_dim=64, qass_mode="full").cuda()
    with torch.no_grad():
        for p in mod.parameters():
            p.add_(torch.randn_like(p) * 0.2)
    params = _qass_params(mod)
    E = H * D
    base = torch.randn(R, 3 * E, device="cuda").to(torch.bfloat16)
    q = base[:, E:2 * E]
    dq_out = torch.randn(R, E, device="cuda")
    monkeypatch.setenv("NORI_QASS_TC", "1")
    out, dq, grads = _run(params, q, H, D, dq_out)
    monkeypatch.setenv("NORI_QASS_TC", "0")
    out0, dq0, grads0 = _run(params, q, H, D, dq_out)
    from synthefy_nori_b200 import ops

    ops.check_status(q.device)
    # forward: both kernels run the gate MLP on bf16 operands with fp32 accumulation
    assert _rel(out, out0) < 1e-2
    ref = _qass_apply_torch(params, "full", q, 777, H, D)
    assert _rel(out, ref) < 1e-2
    # backward against the legacy kernel and the fp32 statement
    assert _rel(dq, dq0) < 1e-2
    qf = q.float().clone().requires_grad_(True)
    for p in params:
        if p is not None:
            p.grad = None
    with torch.enable_grad():
        _qass_apply_torch(params, "full", qf, 777, H, D).backward(dq_out)
    assert _rel(dq, qf.grad) < 2e-2
    for p, gk, g0 in zip(params, grads, grads0):
        if p is None or p.grad is None:
            continue
        assert _rel(gk, g0) < 3e-2, (p.shape, _rel(gk, g0))
        cos = torch.nn.functional.cosine_similarity(gk.flatten().double(), p.grad.flatten().double(), dim=0)
        assert cos > 0.99, (p.shape, float(cos))


def test_qass_tc_writes_into_strided_gradient_block(monkeypatch):
    monkeypatch.setenv("NORI_QASS_TC", "1")
    H, D, R = 8, 56, 1000
    torch.manual_seed(3)
    mod = QASSMaxScaling(num_heads=H, head_dim=D, hidden_dim=64, qass_mode="full").cuda()
    params = _qass_params(mod)
    E = H * D
    q = torch.randn(R, 5 * E, device="cuda").to(torch.bfloat16)[:, :E]
    dq_out = torch.randn(R, E, device="cuda")
    g = Geometry(B=1, ep=99, nq=0, T=1, E=E, H=H)
    dq, _ = _qass_backward(params, "full", q, 99, g, dq_out)
    wide = torch.zeros(R, 5 * E, device="cuda", dtype=torch.bfloat16)
    _qass_backward(params, "full", q, 99, g, dq_out, out=wide[:, :E])
    assert torch.equal(wide[:, :E], dq)
    assert wide[:, E:].abs().max().item() == 0
