"""tcgen05 GEMM family vs an fp32 PyTorch reference of the same op."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from synthefy_nori_b200 import ops  # noqa: E402


def _ref(a, w):
    return a.float() @ w.float().T


def _rand(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (300, 448, 448), (1000, 1344, 448), (257, 96, 128), (4096, 896, 896), (77, 352, 352)])
@pytest.mark.parametrize("bn", [0, 128, 192, 256])
def test_gemm_plain(M, N, K, bn):
    torch.manual_seed(0)
    a, w = _rand(M, K), _rand(N, K, scale=K ** -0.5)
    rs = torch.rand(M, device="cuda") + 0.5
    bias = torch.randn(N, device="cuda")
    out = ops.gemm(a, w, rs, bias, bn=bn)
    ref = _ref(a, w) * rs[:, None] + bias
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
    ops.check_status(a.device)


def test_gemm_strided_a():
    torch.manual_seed(1)
    big = _rand(513, 3 * 448)
    a = big[:, 448:896]  # row stride 1344
    w = _rand(448, 448, scale=448 ** -0.5)
    out = ops.gemm(a, w)
    torch.testing.assert_close(out.float(), _ref(a, w), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("M,E,H", [(500, 448, 896), (129, 128, 256)])
def test_gemm_swiglu(M, E, H):
    torch.manual_seed(2)
    a = _rand(M, E)
    wg, wu = _rand(H, E, scale=E ** -0.5), _rand(H, E, scale=E ** -0.5)
    rs = torch.rand(M, device="cuda") + 0.5
    out = ops.gemm_swiglu(a, ops.interleave_swiglu_weights(wg, wu), rs)
    g = _ref(a, wg) * rs[:, None]
    u = _ref(a, wu) * rs[:, None]
    ref = torch.nn.functional.silu(g) * u
    torch.testing.assert_close(out.float(), ref, atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("M,E,H", [(500, 448, 1344), (129, 128, 256), (1000, 352, 704)])
@pytest.mark.parametrize("bn", [0, 128, 256])
def test_gemm_swiglu_bwd(M, E, H, bn):
    """Gradient of the SwiGLU pre-activation from one GEMM (recomputed gate / up, dh read by
    the epilogue) against autograd of the fp32 statement."""
    torch.manual_seed(3)
    a = _rand(M, E)
    wg, wu = _rand(H, E, scale=E ** -0.5), _rand(H, E, scale=E ** -0.5)
    rs = torch.rand(M, device="cuda") + 0.5
    dh = _rand(M, H)
    out = ops.gemm_swiglu_bwd(a, ops.interleave_swiglu_weights(wg, wu), dh, row_scale=rs, bn=bn)
    g = (_ref(a, wg) * rs[:, None]).requires_grad_()
    u = (_ref(a, wu) * rs[:, None]).requires_grad_()
    (torch.nn.functional.silu(g) * u).backward(dh.float())
    ref = torch.stack((g.grad, u.grad), 2).reshape(M, 2 * H)
    torch.testing.assert_close(out.float(), ref, atol=3e-2, rtol=3e-2)
    ops.check_status(a.device)


@pytest.mark.parametrize("M,N,K", [(700, 448, 896), (64, 128, 128)])
def test_gemm_residual(M, N, K):
    torch.manual_seed(3)
    a, w, r = _rand(M, K), _rand(N, K, scale=K ** -0.5), _rand(M, N)
    ssq = torch.zeros(M, device="cuda")
    out = ops.gemm_residual(a, w, r, 0.25, ssq)
    ref = r.float() + 0.25 * _ref(a, w)
    torch.testing.assert_close(out.float(), ref, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(ssq, (out.float() ** 2).sum(1), atol=1e-2, rtol=1e-3)


@pytest.mark.parametrize("M,N,K", [(1000, 448, 1344), (300, 896, 448), (129, 128, 256)])
def test_gemm_dgrad_w_kn(M, N, K):
    """dX = dY @ W with W [N_in... stored [K, N]]: B operand read MN-major."""
    torch.manual_seed(4)
    dy = _rand(M, K)
    w = _rand(K, N, scale=K ** -0.5)  # W stored [K, N]
    out = ops.gemm(dy, w, w_kn=True)
    torch.testing.assert_close(out.float(), dy.float() @ w.float(), atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("T,No,Ki", [(5000, 448, 448), (777, 1344, 448), (64, 128, 256)])
def test_gemm_wgrad(T, No, Ki):
    torch.manual_seed(5)
    dy, x = _rand(T, No, scale=0.1), _rand(T, Ki)
    out = torch.randn(No, Ki, device="cuda")
    ref = out + dy.float().T @ x.float()
    ops.gemm_wgrad(dy, x, out)
    torch.testing.assert_close(out, ref, atol=5e-2, rtol=1e-2)


def test_gemm_gelu_epilogue_and_backward():
    """Exact GELU in the store epilogue (after the row scale) and the GELU backward kernel,
    against fp32 PyTorch."""
    torch.manual_seed(4)
    a = torch.randn(300, 192, device="cuda").to(torch.bfloat16)
    w = (0.1 * torch.randn(136, 192, device="cuda")).to(torch.bfloat16)
    rs = torch.rand(300, device="cuda") + 0.5
    z = (a.float() @ w.float().t()) * rs[:, None]
    out = ops.gemm(a, w, row_scale=rs, act="gelu")
    torch.testing.assert_close(out.float(), torch.nn.functional.gelu(z), atol=2e-2, rtol=2e-2)
    zb = z.to(torch.bfloat16)
    dh = torch.randn_like(zb)
    zf = zb.float().requires_grad_(True)
    torch.nn.functional.gelu(zf).backward(dh.float())
    torch.testing.assert_close(ops.gelu_bwd(dh, zb).float(), zf.grad, atol=2e-2, rtol=2e-2)
