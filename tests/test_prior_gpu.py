"""SCM-prior kernels (K19) against plain fp32 PyTorch: every activation of ``scm_act``,
the batched noisy linear map of ``scm_linear`` (noise-free values, context-row column
sums, noise moments), and the generators built on them."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

ACTS = {0: torch.tanh, 1: lambda x: torch.nn.functional.leaky_relu(x, 0.01), 2: torch.nn.functional.elu,
        3: lambda x: x, 4: torch.nn.functional.selu, 5: torch.nn.functional.silu, 6: torch.relu,
        7: torch.nn.functional.softplus, 8: torch.nn.functional.relu6, 9: torch.nn.functional.hardtanh,
        10: lambda x: 2 * (x >= 0).float() - 1, 11: lambda x: torch.exp(-x * x), 12: torch.exp,
        13: lambda x: torch.sqrt(x.abs()), 14: lambda x: (x.abs() <= 1).float(), 15: torch.sin,
        16: lambda x: x * x, 17: torch.abs}


def test_scm_act_every_activation():
    from synthefy_nori_b200 import ops

    B, N, H = len(ACTS) + 1, 67, 40
    torch.manual_seed(0)
    h = torch.randn(B, N, H, device="cuda") * 2
    code = torch.arange(B, dtype=torch.int32, device="cuda")  # 0..17 and 18 (random Fourier)
    scale = torch.rand(B, device="cuda") + 0.5
    shift = torch.randn(B, device="cuda") * 0.3
    width = torch.full((B,), 33, dtype=torch.int32, device="cuda")
    mean = torch.randn(B, H, device="cuda") * 0.1
    rstd = torch.rand(B, H, device="cuda") + 0.5
    rff = torch.zeros(B, 3, 256, device="cuda")
    rff[-1, 0] = torch.rand(256, device="cuda") * 20
    rff[-1, 1] = torch.rand(256, device="cuda") * 6.28
    rff[-1, 2] = torch.randn(256, device="cuda") / 16
    out = ops.lib().scm_act(h, code, scale, shift, width, mean, rstd, rff)
    z = (h - mean.unsqueeze(1)) * rstd.unsqueeze(1)
    for b in range(B):
        if b in ACTS:
            ref = ACTS[b](scale[b] * (z[b] + shift[b]))
        else:
            ref = (rff[b, 2] * torch.sin(rff[b, 0] * z[b].unsqueeze(-1) + rff[b, 1])).sum(-1)
        ref = torch.where(torch.isfinite(ref), ref, torch.zeros_like(ref))
        torch.testing.assert_close(out[b, :, :33], ref[:, :33], atol=1e-4, rtol=1e-4, msg=f"act {b}")
        assert bool((out[b, :, 33:] == 0).all())


def test_scm_linear_values_sums_and_noise():
    from synthefy_nori_b200 import ops

    torch.manual_seed(1)
    B, N, K, H = 3, 300, 70, 96
    A = torch.randn(B, N, K, device="cuda")
    W = torch.randn(B, H, K, device="cuda") / math.sqrt(K)
    bias = torch.randn(B, H, device="cuda") * 0.1
    width = torch.tensor([96, 50, 0], dtype=torch.int32, device="cuda")
    zero = torch.zeros(B, H, device="cuda")
    cs = torch.zeros(B, H, device="cuda", dtype=torch.float64)
    cq = torch.zeros_like(cs)
    out = ops.lib().scm_linear(A, W, bias, zero, width, 200, 7, 1, cs, cq)
    ref = (torch.bmm(A, W.transpose(1, 2)) + bias.unsqueeze(1)).clamp(-100, 100)
    for b, w in enumerate([96, 50, 0]):
        torch.testing.assert_close(out[b, :, :w], ref[b, :, :w], atol=1e-4, rtol=1e-4)
        assert bool((out[b, :, w:] == 0).all())
        torch.testing.assert_close(cs[b, :w].float(), ref[b, :200, :w].sum(0), atol=1e-3, rtol=1e-4)
        torch.testing.assert_close(cq[b, :w].float(), (ref[b, :200, :w] ** 2).sum(0), atol=1e-2, rtol=1e-4)
    # noise: N(0, sigma^2) draws, independent across elements
    sig = torch.full((B, H), 0.5, device="cuda")
    Wz = torch.zeros_like(W)
    cs.zero_()
    cq.zero_()
    big = torch.zeros(B, 4000, K, device="cuda")
    noise = ops.lib().scm_linear(big, Wz, zero, sig, torch.full((B,), H, dtype=torch.int32, device="cuda"), 4000,
                                 11, 2, cs, cq)
    assert abs(float(noise.mean())) < 5e-3 and abs(float(noise.std()) - 0.5) < 5e-3
    again = ops.lib().scm_linear(big, Wz, zero, sig, torch.full((B,), H, dtype=torch.int32, device="cuda"), 4000,
                                 11, 2, cs, cq)
    assert torch.equal(noise, again)  # a pure function of (seed, layer, position)


def test_priors_produce_standardised_tables():
    from synthefy_nori_b200.training.prior import PriorConfig, scm_prior_batch
    from synthefy_nori_b200.training.scm_prior import scm_prior_tables

    dev = torch.device("cuda")
    b = scm_prior_batch(PriorConfig(max_features=20, pad_features=20), 6, 300, 200, seed=3, device=dev)
    assert b.x.shape == (6, 300, 20) and torch.isfinite(b.x).all() and torch.isfinite(b.y).all()
    torch.testing.assert_close(b.y[:, :200].mean(1), torch.zeros(6, device=dev), atol=1e-4, rtol=0)
    X, y, meta = scm_prior_tables(12, 256, [5, 9, 20, 3, 50, 7, 11, 2, 30, 8, 13, 40], 180, seed=5, device=dev,
                                  pad_features=50)
    assert X.shape == (12, 256, 50) and torch.isfinite(X).all() and torch.isfinite(y).all()
    assert set(meta["scm_type"]) <= {"mlp", "tree"}
    ys = y[:, :180].std(1, unbiased=False)
    assert bool(((ys - 1).abs() < 1e-3).all())
