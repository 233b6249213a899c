"""tcgen05 flash attention forward vs an fp32 PyTorch reference (small shapes first)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from synthefy_nori_b200 import ops  # noqa: E402


def _ref(q, k, v, scale):
    s = torch.einsum("bqd,bkd->bqk", q.float(), k.float()) * scale
    return torch.einsum("bqk,bkd->bqd", torch.softmax(s, -1), v.float()), torch.logsumexp(s, -1)


@pytest.mark.parametrize("BH,Nq,Nk,D", [(1, 128, 128, 64), (2, 100, 37, 56), (3, 300, 700, 56), (2, 129, 257, 64)])
def test_tc_headmajor(BH, Nq, Nk, D):
    torch.manual_seed(0)
    q = torch.randn(BH, Nq, D, device="cuda").to(torch.bfloat16)
    k = torch.randn(BH, Nk, D, device="cuda").to(torch.bfloat16)
    v = torch.randn(BH, Nk, D, device="cuda").to(torch.bfloat16)
    o = torch.zeros(BH, Nq, D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(BH, Nq, device="cuda")
    lay = lambda n: (n * D, 0, 0, D, 1, 1)  # noqa: E731
    ops.attention_fwd_tc(q, k, v, o, lq=lay(Nq), lk=lay(Nk), lv=lay(Nk), lo=lay(Nq), BH=BH, Nq=Nq, Nk=Nk, d=D,
                         scale=1 / math.sqrt(D), lse=lse)
    ops.check_status(q.device)
    ref, rl = _ref(q, k, v, 1 / math.sqrt(D))
    torch.testing.assert_close(o.float(), ref, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(lse, rl, atol=2e-3, rtol=2e-3)


def test_tc_token_major_sequence_layout():
    torch.manual_seed(1)
    B, N, T, H, D = 2, 150, 5, 8, 56
    E = H * D
    y = torch.randn(B * N * T, 5 * E, device="cuda").to(torch.bfloat16)  # [.., (q k v k2 v2)]
    q = torch.randn(B * N * T, E, device="cuda").to(torch.bfloat16)
    o = torch.zeros(B * N * T, E, device="cuda", dtype=torch.bfloat16)
    lq = (N * T * E, E, D, T * E, T, H)
    l5 = (N * T * 5 * E, 5 * E, D, T * 5 * E, T, H)
    ops.attention_fwd_tc(q, y[:, E:2 * E], y[:, 2 * E:3 * E], o, lq=lq, lk=l5, lv=l5, lo=lq, BH=B * T * H, Nq=N, Nk=N,
                         d=D, scale=D ** -0.5)
    ops.check_status(q.device)
    qs = q.view(B, N, T, H, D).permute(0, 2, 3, 1, 4).reshape(-1, N, D)
    ks = y[:, E:2 * E].reshape(B, N, T, H, D).permute(0, 2, 3, 1, 4).reshape(-1, N, D)
    vs = y[:, 2 * E:3 * E].reshape(B, N, T, H, D).permute(0, 2, 3, 1, 4).reshape(-1, N, D)
    ref, _ = _ref(qs, ks, vs, D ** -0.5)
    ref = ref.view(B, T, H, N, D).permute(0, 3, 1, 2, 4).reshape(B * N * T, E)
    torch.testing.assert_close(o.float(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("BH,Nq,Nk,D", [(1, 128, 128, 64), (2, 100, 37, 56), (3, 300, 260, 56), (2, 129, 257, 64)])
def test_tc_backward_matches_reference(BH, Nq, Nk, D):
    torch.manual_seed(1)
    scale = 1 / math.sqrt(D)
    q = torch.randn(BH, Nq, D, device="cuda").to(torch.bfloat16)
    k = torch.randn(BH, Nk, D, device="cuda").to(torch.bfloat16)
    v = torch.randn(BH, Nk, D, device="cuda").to(torch.bfloat16)
    o = torch.empty(BH, Nq, D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(BH, Nq, device="cuda")
    lay = lambda n: (n * D, 0, 0, D, 1, 1)  # noqa: E731
    ops.attention_fwd_tc(q, k, v, o, lq=lay(Nq), lk=lay(Nk), lv=lay(Nk), lo=lay(Nq), BH=BH, Nq=Nq, Nk=Nk, d=D,
                         scale=scale, lse=lse)
    do = torch.randn(BH, Nq, D, device="cuda").to(torch.bfloat16)
    dq = torch.zeros(BH, Nq, D, device="cuda")
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    ops.attention_bwd_tc(q, k, v, o, do, lse, dq, dk, dv, lq=lay(Nq), lkv=lay(Nk), lo=lay(Nq), ldo=lay(Nq),
                         ldkv=lay(Nk), ldq=lay(Nq), BH=BH, Nq=Nq, Nk=Nk, d=D, scale=scale)
    ops.check_status(q.device)
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    ref, _ = _ref(qf, kf, vf, scale)
    ref.backward(do.float())
    for got, want in ((dq, qf.grad), (dk.float(), kf.grad), (dv.float(), vf.grad)):
        rel = ((got - want).norm() / want.norm()).item()
        assert rel < 2e-2, rel


def test_exp2_poly_against_exp2f():
    """The softmax's FMA-pipe 2^x (minimax cubic + exponent-field add) against CUDA's
    exp2f over its whole input range [-125, 0]: relative error within the stated 7.5e-5."""
    from synthefy_nori_b200 import ops

    x = torch.linspace(-125.0, 0.0, 2_000_001, device="cuda")
    x = torch.cat([x, -torch.rand(1_000_000, device="cuda") * 3.0, torch.tensor([-0.5, -0.25, -1e-7, 0.0],
                                                                                device="cuda")])
    got = ops.lib().exp2_poly_eval(x.contiguous())
    ref = torch.exp2(x)  # CUDA exp2f
    rel = ((got.double() - ref.double()) / ref.double()).abs()
    assert float(rel.max()) <= 7.6e-5
    exact = torch.exp2(x.double())
    assert float(((got.double() - exact) / exact).abs().max()) <= 7.6e-5
