"""The native regression head + pinball objective against the fp32 PyTorch modules:
LayerNorm+activation kernels (strided rows), bias-gradient column sums, and the whole
head/loss node (value and every parameter / input gradient)."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("act", [0, 1, 2])
@pytest.mark.parametrize("C", [64, 1344, 2048])
def test_ln_act_fwd_bwd(act, C):
    from synthefy_nori_b200 import ops

    lib = ops.lib()
    torch.manual_seed(act * 7 + C)
    R = 333
    base = torch.randn(R, C + 16, device="cuda") * 3 + 1
    x = base.to(torch.bfloat16)[:, 8 : 8 + C]  # strided rows
    g = torch.randn(C, device="cuda")
    b = torch.randn(C, device="cuda")
    y, mean, rstd = lib.ln_act_fwd(x, g, b, 1e-5, act)
    xf = x.float().requires_grad_(True)
    gf, bf = g.clone().requires_grad_(True), b.clone().requires_grad_(True)
    z = F.layer_norm(xf, (C,), gf, bf, 1e-5)
    ref = {0: lambda t: t, 1: F.gelu, 2: F.relu}[act](z)
    torch.testing.assert_close(y.float(), ref, atol=3e-2, rtol=2e-2)
    dy = torch.randn(R, C, device="cuda").to(torch.bfloat16)
    ref.backward(dy.float())
    dx = torch.empty(R, C + 8, device="cuda", dtype=torch.bfloat16)[:, :C]
    dg = torch.zeros(C, device="cuda")
    db = torch.zeros(C, device="cuda")
    lib.ln_act_bwd(dy, x, g, b, mean, rstd, act, dx, dg, db)
    torch.testing.assert_close(dx.float(), xf.grad, atol=5e-2, rtol=3e-2)
    torch.testing.assert_close(dg, gf.grad, atol=5e-2 * R ** 0.5, rtol=2e-2)
    torch.testing.assert_close(db, bf.grad, atol=5e-2 * R ** 0.5, rtol=2e-2)


def test_colsum():
    from synthefy_nori_b200 import ops

    y = torch.randn(1000, 1008, device="cuda").to(torch.bfloat16)
    out = torch.ones(999, device="cuda")
    ops.lib().colsum_bf16(y, out)
    torch.testing.assert_close(out, 1 + y.float()[:, :999].sum(0), atol=1e-2, rtol=1e-4)


@pytest.mark.parametrize("preset", ["nori-tiny", "nori-6m"])
def test_head_pinball_matches_torch(preset):
    from synthefy_nori_b200.models.config import preset_config
    from synthefy_nori_b200.ops.head import head_pinball_loss, head_supported
    from synthefy_nori_b200.training.loss import pinball_objective_torch
    from synthefy_nori_b200.utils.loading import build_model

    torch.manual_seed(0)
    model = build_model(preset_config(preset)).cuda()
    assert head_supported(model)
    E = model.reg_y_decoder[0].in_features
    B, nq, T = 3, 57, 5
    X = (torch.randn(B * nq, T, E, device="cuda") * 0.5).to(torch.bfloat16).requires_grad_(True)
    last = X[:, -1]
    target = torch.randn(B, nq, device="cuda")
    q = torch.tensor(model.regression_quantiles, device="cuda")
    loss = head_pinball_loss(model, last, target, q, 0.0, 0.05, 0.0)
    params = [p for p in list(model.encoder_out_norm.parameters()) + list(model.reg_y_decoder.parameters())]
    grads = torch.autograd.grad(loss, [X] + params)
    # fp32 oracle on the same (bf16-valued) inputs, and the same module under bf16
    # autocast (the precision the PyTorch path trains at): the native node must be within
    # twice the autocast path's own error of the fp32 oracle (relative L2 per tensor)
    def torch_grads(autocast):
        Xr = X.detach().float().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            pred = model.reg_y_decoder(model.encoder_out_norm(Xr[:, -1])).view(B, nq, -1)
        ref = pinball_objective_torch(pred.float(), target, q, 0.0, 0.05, 0.0)
        return ref, torch.autograd.grad(ref, [Xr] + params)

    ref, rgrads = torch_grads(False)
    _, agrads = torch_grads(True)
    torch.testing.assert_close(loss.float(), ref.float(), atol=2e-3, rtol=1e-2)
    for gn, gr, ga in zip(grads, rgrads, agrads):
        err = float((gn.float() - gr).norm() / (gr.norm() + 1e-30))
        base = float((ga.float() - gr).norm() / (gr.norm() + 1e-30))
        assert err <= max(2 * base, 1e-2), (gn.shape, err, base)
