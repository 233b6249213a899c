"""tcgen05 feature (within-row) attention against an fp32 PyTorch reference, read straight
from a token-major fused QKV buffer ``[rows * T, 3 * H * Dp]`` (the projection GEMM's
output) and written to a token-major ``[rows * T, H * Dp]`` output; odd row counts (the
last item's second row does not exist), short rows and the 64-token limit."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from synthefy_nori_b200 import ops  # noqa: E402


def _layouts(T, H, Dp):
    A = H * Dp
    return (T * 3 * A, 0, Dp, 3 * A, 1, H), (T * A, 0, Dp, A, 1, H)


def _qkv(n_rows, T, H, D, Dp, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    y = torch.zeros(n_rows * T, 3, H, Dp, device="cuda")
    y[..., :D] = torch.randn(n_rows * T, 3, H, D, device="cuda", generator=g)
    return y.reshape(n_rows * T, 3 * H * Dp).to(torch.bfloat16)


def _ref(y, n_rows, T, H, D, Dp, scale):
    y4 = y.float().view(n_rows, T, 3, H, Dp)[..., :D]
    q, k, v = (y4[:, :, i].permute(0, 2, 1, 3) for i in range(3))  # [rows, H, T, D]
    s = torch.einsum("rhqd,rhkd->rhqk", q, k) * scale
    o = torch.einsum("rhqk,rhkd->rhqd", torch.softmax(s, -1), v)
    return o, torch.logsumexp(s, -1)


@pytest.mark.parametrize("n_rows,T,H,D", [(37, 51, 8, 56), (6, 64, 2, 56), (5, 7, 3, 44), (1, 1, 1, 64), (300, 33, 8, 48)])
def test_feature_attention_fwd_tc(n_rows, T, H, D):
    Dp = -(-D // 8) * 8
    A = H * Dp
    scale = 1 / math.sqrt(D)
    y = _qkv(n_rows, T, H, D, Dp, seed=n_rows + T)
    l3, l1 = _layouts(T, H, Dp)
    o = torch.full((n_rows * T, A), 7.0, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(n_rows * H, T, device="cuda")
    assert ops.feat_tc_supported(T, Dp)
    ops.attention_feat_fwd_tc(y[:, :A], y[:, A : 2 * A], y[:, 2 * A :], o, lq=l3, lk=l3, lv=l3, lo=l1,
                              BH=n_rows * H, T=T, d=Dp, scale=scale, lse=lse)
    ops.check_status(torch.device("cuda"))
    ref, ref_lse = _ref(y, n_rows, T, H, D, Dp, scale)
    got = o.float().view(n_rows, T, H, Dp).permute(0, 2, 1, 3)
    torch.testing.assert_close(got[..., :D], ref, atol=2e-2, rtol=2e-2)
    if Dp > D:
        assert got[..., D:].abs().max().item() == 0  # zero padding columns stay zero
    torch.testing.assert_close(lse.view(n_rows, H, T), ref_lse, atol=1e-3, rtol=1e-3)


def test_feature_attention_fwd_tc_matches_mma_kernel():
    """Same output as the mma.sync feature-attention kernel on the training shape."""
    n_rows, T, H, D = 401, 51, 8, 56
    A = H * D
    y = _qkv(n_rows, T, H, D, D, seed=3)
    l3, l1 = _layouts(T, H, D)
    o1 = torch.empty(n_rows * T, A, device="cuda", dtype=torch.bfloat16)
    o2 = torch.empty_like(o1)
    lse1 = torch.empty(n_rows * H, T, device="cuda")
    lse2 = torch.empty_like(lse1)
    kw = dict(lq=l3, lk=l3, lv=l3, lo=l1, BH=n_rows * H, d=D, scale=1 / math.sqrt(D))
    ops.attention_fwd(y[:, :A], y[:, A : 2 * A], y[:, 2 * A :], o1, Nq=T, Nk=T, lse=lse1, **kw)
    ops.attention_feat_fwd_tc(y[:, :A], y[:, A : 2 * A], y[:, 2 * A :], o2, T=T, lse=lse2, **kw)
    torch.testing.assert_close(o2.float(), o1.float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(lse2, lse1, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("n_rows,T,H,D", [(37, 51, 8, 56), (6, 64, 2, 56), (5, 7, 3, 44), (1, 1, 1, 64), (300, 33, 8, 48)])
def test_feature_attention_bwd_tc(n_rows, T, H, D):
    Dp = -(-D // 8) * 8
    A = H * Dp
    scale = 1 / math.sqrt(D)
    y = _qkv(n_rows, T, H, D, Dp, seed=2 * n_rows + T)
    l3, l1 = _layouts(T, H, Dp)
    o = torch.empty(n_rows * T, A, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(n_rows * H, T, device="cuda")
    ops.attention_feat_fwd_tc(y[:, :A], y[:, A : 2 * A], y[:, 2 * A :], o, lq=l3, lk=l3, lv=l3, lo=l1,
                              BH=n_rows * H, T=T, d=Dp, scale=scale, lse=lse)
    g = torch.Generator(device="cuda").manual_seed(7)
    do = torch.zeros(n_rows * T, H, Dp, device="cuda")
    do[..., :D] = torch.randn(n_rows * T, H, D, device="cuda", generator=g)
    do = do.reshape(n_rows * T, A).to(torch.bfloat16)
    dy = torch.full((n_rows * T, 3 * A), 5.0, device="cuda", dtype=torch.bfloat16)
    ops.attention_feat_bwd_tc(y[:, :A], y[:, A : 2 * A], y[:, 2 * A :], o, do, lse, dy[:, :A], dy[:, A : 2 * A],
                              dy[:, 2 * A :], lq=l3, lkv=l3, lo=l1, lg=l3, BH=n_rows * H, T=T, d=Dp, scale=scale)
    ops.check_status(torch.device("cuda"))
    yf = y.float().requires_grad_(True)
    ref, _ = _ref(yf, n_rows, T, H, D, Dp, scale)
    ref.backward(do.float().view(n_rows, T, H, Dp)[..., :D].permute(0, 2, 1, 3))
    got = dy.float().view(n_rows * T, 3, H, Dp)
    want = yf.grad.view(n_rows * T, 3, H, Dp)
    for i, name in enumerate("qkv"):
        torch.testing.assert_close(got[:, i, :, :D], want[:, i, :, :D], atol=5e-2, rtol=5e-2, msg=lambda m: f"d{name}: {m}")
    if Dp > D:
        assert got[..., D:].abs().max().item() == 0  # zero padding columns of the heads stay zero


def test_feature_attention_bwd_tc_matches_mma_kernel():
    """Same gradients as the mma.sync single-tile backward on the training shape."""
    n_rows, T, H, D = 401, 51, 8, 56
    A = H * D
    scale = 1 / math.sqrt(D)
    y = _qkv(n_rows, T, H, D, D, seed=5)
    l3, l1 = _layouts(T, H, D)
    o = torch.empty(n_rows * T, A, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(n_rows * H, T, device="cuda")
    ops.attention_fwd(y[:, :A], y[:, A : 2 * A], y[:, 2 * A :], o, lq=l3, lk=l3, lv=l3, lo=l1, BH=n_rows * H, Nq=T,
                      Nk=T, d=D, scale=scale, lse=lse)
    do = (0.5 * torch.randn(n_rows * T, A, device="cuda")).to(torch.bfloat16)
    dy1 = torch.empty(n_rows * T, 3 * A, device="cuda", dtype=torch.bfloat16)
    dy2 = torch.empty_like(dy1)
    ops.attention_bwd(y[:, :A], y[:, A : 2 * A], y[:, 2 * A :], o, do, lse, None, dy1[:, A : 2 * A], dy1[:, 2 * A :],
                      lq=l3, lk=l3, lv=l3, lo=l1, ldo=l1, ldk=l3, ldv=l3, ldq=l3, BH=n_rows * H, Nq=T, Nk=T, d=D,
                      scale=scale, dq_bf16=dy1[:, :A])
    ops.attention_feat_bwd_tc(y[:, :A], y[:, A : 2 * A], y[:, 2 * A :], o, do, lse, dy2[:, :A], dy2[:, A : 2 * A],
                              dy2[:, 2 * A :], lq=l3, lkv=l3, lo=l1, lg=l3, BH=n_rows * H, T=T, d=D, scale=scale)
    torch.testing.assert_close(dy2.float(), dy1.float(), atol=2e-2, rtol=2e-2)
