"""Fused QASS rescale (forward / backward) vs its fp32 PyTorch statement."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from synthefy_nori_b200.models.layers import QASSMaxScaling  # noqa: E402
from synthefy_nori_b200.ops.fused_layer import Geometry, _qass_apply, _qass_apply_torch, _qass_backward, _qass_params  # noqa: E402


@pytest.mark.parametrize("mode", ["full", "base_only", "log_only"])
@pytest.mark.parametrize("H,D", [(8, 56), (2, 64)])
def test_qass_fused_matches_torch(mode, H, D):
    torch.manual_seed(0)
    mod = QASSMaxScaling(num_heads=H, head_dim=D, hidden_dim=64, qass_mode=mode).cuda()
    with torch.no_grad():
        for p in mod.parameters():
            p.add_(torch.randn_like(p) * 0.2)
    params = _qass_params(mod)
    R, E = 333, H * D
    base = torch.randn(R, 3 * E, device="cuda").to(torch.bfloat16)
    q = base[:, E:2 * E]  # row-strided view, as in the layer
    out = _qass_apply(params, mode, q, 777, H, D)
    ref = _qass_apply_torch(params, mode, q, 777, H, D)
    # bf16 gate MLP (the reference runs it under bf16 autocast): almost all elements within
    # bf16 tolerance, none far off
    bad = ((out.float() - ref).abs() > 3e-2 + 3e-2 * ref.abs()).float().mean().item()
    assert bad < 1e-3, bad
    assert (out.float() - ref).abs().max().item() < 0.08 * ref.abs().max().item()
    # backward
    dq_out = torch.randn(R, E, device="cuda")
    g = Geometry(B=1, ep=777, nq=0, T=1, E=E, H=H)
    dq, grads = _qass_backward(params, mode, q, 777, g, dq_out)
    qf = q.float().clone().requires_grad_(True)
    ps = [p for p in params if p is not None]
    for p in ps:
        p.grad = None
    with torch.enable_grad():
        r2 = _qass_apply_torch(params, mode, qf, 777, H, D)
        r2.backward(dq_out)
    # bf16 operands in the gate-MLP backward: compare in norm
    rel = ((dq.float() - qf.grad).norm() / qf.grad.norm()).item()
    assert rel < 2e-2, rel
    for p, gk in zip(params, grads):
        if p is None or p.grad is None:
            continue
        assert gk is not None
        cos = torch.nn.functional.cosine_similarity(gk.flatten().double(), p.grad.flatten().double(), dim=0)
        assert cos > 0.99, (p.shape, float(cos))
    # the same gradient written in place into a column block of a wider buffer
    wide = torch.zeros(R, 3 * E, device="cuda", dtype=torch.bfloat16)
    _qass_backward(params, mode, q, 777, g, dq_out, out=wide[:, E:2 * E])
    assert torch.equal(wide[:, E:2 * E], dq)
    assert wide[:, :E].abs().max().item() == 0 and wide[:, 2 * E:].abs().max().item() == 0
