"""Memory-bound kernels vs fp32 PyTorch references."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from synthefy_nori_b200 import ops  # noqa: E402


def test_rms_scale():
    x = torch.randn(1000, 448, device="cuda").to(torch.bfloat16)
    rs = ops.rms_scale(x, 1e-5)
    ref = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-5)
    torch.testing.assert_close(rs, ref, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_pinball_matches_autograd(dtype):
    torch.manual_seed(0)
    B, nq, K = 3, 17, 999
    q = torch.tensor([(i + 1) / 1000 for i in range(K)], device="cuda")
    pred = (torch.randn(B, nq, K, device="cuda").sort(-1).values + 0.05 * torch.randn(B, nq, K, device="cuda")).to(dtype)
    target = torch.randn(B, nq, device="cuda")
    var = target.var(dim=1, unbiased=False).clamp(min=0.01)
    p = pred.float().clone().requires_grad_(True)
    e = target.unsqueeze(-1) - p
    loss_pin = torch.maximum(q * e, (q - 1) * e).mean(dim=(1, 2))
    diff = p[..., :-1] - p[..., 1:]
    mono = torch.relu(diff).pow(2).mean(-1).mean(1)
    mse = ((p.mean(-1) - target) ** 2).mean(1) / var
    ref = (loss_pin + 0.05 * mono + 0.1 * mse).sum() / B
    ref.backward()
    loss, grad = ops.pinball_loss_grad(pred.view(-1, K).contiguous(), target.reshape(-1).contiguous(), q, (1.0 / var).contiguous(), nq,
                                       0.0, 0.05, 0.1)
    torch.testing.assert_close(loss[0], ref.detach(), atol=1e-4, rtol=1e-4)
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    torch.testing.assert_close(grad.float().view(B, nq, K), p.grad, atol=tol, rtol=tol)


def test_adamw_ema_matches_torch():
    torch.manual_seed(1)
    n = 10007
    p0 = torch.randn(n, device="cuda")
    ref_p = torch.nn.Parameter(p0.clone())
    opt = torch.optim.AdamW([ref_p], lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01)
    p, m, v, ema = p0.clone(), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda"), p0.clone()
    ref_ema = p0.clone()
    pbf = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    for step in range(1, 4):
        g = torch.randn(n, device="cuda") * 3
        ref_p.grad = g.clone()
        torch.nn.utils.clip_grad_norm_([ref_p], 1.0)
        opt.step()
        ref_ema.mul_(0.999).add_(ref_p.detach(), alpha=0.001)
        nsq = torch.zeros(1, device="cuda")
        ops.grad_sumsq(g, nsq)
        ops.adamw_ema_step(p, g, m, v, lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, wd=0.01, step=step, ema=ema,
                           p_bf16=pbf, norm_sq=nsq, ema_decay=0.999, max_norm=1.0)
    torch.testing.assert_close(p, ref_p.detach(), atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(ema, ref_ema, atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(pbf.float(), p, atol=1e-2, rtol=1e-2)


def test_quantize_int8_bit_exact():
    x = torch.randn(64, 7, 2, 3, 56, device="cuda")
    q, s = ops.quantize_int8(x)
    scale = x.abs().amax(dim=-1, keepdim=True).clamp_min(1e-12) / 127.0
    qref = torch.clamp(torch.round(x / scale), -127, 127).to(torch.int8)
    assert torch.equal(q, qref)
    torch.testing.assert_close(s, scale, atol=0, rtol=0)


def test_dequantize_int8_bit_exact():
    x = torch.randn(300, 2, 8, 56, device="cuda")
    q, s = ops.quantize_int8(x)
    out = ops.dequantize_int8(q.view(300, -1), s.view(300, -1))
    ref = (q.float() * s).to(torch.bfloat16).view(300, -1)
    assert out.dtype == torch.bfloat16 and torch.equal(out, ref)
