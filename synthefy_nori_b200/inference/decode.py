"""Point estimates from a predicted distribution, on the device.

Parity target: reference ``inference/predictor.py:885-1133`` (quantile-bank collapse
strategies and bar-distribution decode) and ``model/quantile_dist.py:69-208`` (the
trapezoid mean of the piecewise-linear quantile function, with or without exponential
tails).  All strategies run as batched tensor code on the bank's device; the default
``"mean"`` on CUDA uses the fused sort + trapezoid kernel (``ops.quantile_decode``).

Strategies for a bank ``q [N, K]`` at levels ``tau [K]``:

- ``mean`` / ``qdist_simple``: sort, then ``tau_0 q_0 + sum 0.5 (q_i+q_{i+1}) dtau_i +
  (1 - tau_{K-1}) q_{K-1}`` (the mean of the distribution whose quantile function is the
  linear interpolant, constant beyond the outer levels).
- ``qdist``: the same middle area with exponential tails
  ``q(tau) = q_0 + lam_L log(tau/tau_0)`` below ``tau_0`` (area ``tau_0 (q_0 - lam_L)``)
  and ``q(tau) = q_last + lam_R log((1-tau_last)/(1-tau))`` above (area
  ``(1-tau_last)(q_last + lam_R)``); each ``lam`` is the slope of q against the log level
  over the outer ``min(20, K//4)`` quantiles, clamped at 0; non-finite tails fall back to
  the constant ends.
- ``median``: the middle level (mean of the two middle ones for even K).
- ``trimmed_mean``: drop ``max(1, 5% of K)`` levels at each end (at most ``(K-1)//2``).
- ``huber_mean``: Huber weights (k = 1.5) around the middle value with the MAD as scale.
- ``tail_aware``: the mean, except rows whose spread exceeds 1.5x the batch median and
  whose median-to-tail distance on one side is 3x the other side's take that side's outer
  quantile (levels ~0.01 / ~0.99).
"""

from __future__ import annotations

import torch

COLLAPSE_MODES = ("mean", "median", "trimmed_mean", "huber_mean", "tail_aware", "qdist", "qdist_simple")
BAR_ESTIMATORS = ("mean", "mode", "median")


def _trapezoid_mean(q: torch.Tensor, tau: torch.Tensor) -> torch.Tensor:
    """Mean of the sorted bank ``q`` (fp32 or fp64) with constant ends."""
    mid = (0.5 * (q[:, :-1] + q[:, 1:]) * (tau[1:] - tau[:-1])).sum(-1)
    return tau[0] * q[:, 0] + mid + (1.0 - tau[-1]) * q[:, -1]


def check_taus(tau: torch.Tensor, K: int) -> None:
    if tau.shape != (K,):
        raise ValueError(f"tau must have shape ({K},), got {tuple(tau.shape)}")
    if not bool(torch.isfinite(tau).all()) or bool((tau <= 0).any()) or bool((tau >= 1).any()):
        raise ValueError("tau must be finite levels in (0, 1)")
    if K > 1 and bool((tau[1:] <= tau[:-1]).any()):
        raise ValueError("tau must be strictly increasing")


def quantile_mean(q: torch.Tensor, tau: torch.Tensor, *, tails: bool = False, tail_outer_n: int = 20) -> torch.Tensor:
    """Mean of the distribution described by bank ``q [N, K]`` (fp32 result; fp64 inside
    when ``q`` is fp64)."""
    dt = torch.float64 if q.dtype == torch.float64 else torch.float32
    q = torch.sort(q.to(dt), dim=-1).values
    tau = tau.to(device=q.device, dtype=dt)
    K = q.shape[-1]
    if K == 1:
        return q[:, 0]
    if not tails or K < 8:
        return _trapezoid_mean(q, tau)
    n = min(tail_outer_n, K // 4)
    mid = (0.5 * (q[:, :-1] + q[:, 1:]) * (tau[1:] - tau[:-1])).sum(-1)
    lt = torch.log(tau[:n].clamp_min(1e-12))
    lam_l = ((q[:, n - 1] - q[:, 0]) / (lt[-1] - lt[0]).clamp_min(1e-12)).clamp_min(0)
    rt = torch.log((1.0 - tau[-n:]).clamp_min(1e-12))
    lam_r = ((q[:, -1] - q[:, -n]) / (rt[0] - rt[-1]).clamp_min(1e-12)).clamp_min(0)
    left = tau[0] * (q[:, 0] - lam_l)
    right = (1.0 - tau[-1]) * (q[:, -1] + lam_r)
    left = torch.where(torch.isfinite(left), left, tau[0] * q[:, 0])
    right = torch.where(torch.isfinite(right), right, (1.0 - tau[-1]) * q[:, -1])
    return left + mid + right


def _fast_mean(q: torch.Tensor, tau: torch.Tensor) -> torch.Tensor:
    if q.is_cuda and q.shape[-1] <= 1024:
        from synthefy_nori_b200 import ops

        if ops.native_available():
            lv = torch.tensor([0.5], device=q.device, dtype=torch.float32)
            return ops.quantile_decode(q.float().contiguous(), tau.float().to(q.device), lv, False)[0]
    return quantile_mean(q, tau)


def collapse(q: torch.Tensor, tau: torch.Tensor, mode: str = "mean") -> torch.Tensor:
    """Point estimate per row of ``q [N, K]`` (see the module docstring)."""
    if mode not in COLLAPSE_MODES:
        raise ValueError(f"unknown quantile_collapse {mode!r}; expected one of {COLLAPSE_MODES}")
    if q.dim() == 1:
        q = q.unsqueeze(0)
    K = q.shape[-1]
    check_taus(tau.detach().double().cpu(), K)
    if K == 1:
        return q[:, 0].float()
    if mode in ("mean", "qdist_simple"):
        return _fast_mean(q, tau)
    if mode == "qdist":
        return quantile_mean(q, tau, tails=True).float()
    qf = q.float()
    if mode == "median":
        m = K // 2
        return qf[:, m] if K % 2 else qf[:, m - 1 : m + 1].mean(-1)
    if mode == "trimmed_mean":
        trim = min(max(1, int(K * 0.05)), (K - 1) // 2)
        return qf.mean(-1) if trim == 0 else qf[:, trim : K - trim].mean(-1)
    if mode == "huber_mean":
        qs = torch.sort(qf, dim=-1).values
        center = qs[:, K // 2 : K // 2 + 1]
        mad = (qs - center).abs().median(dim=-1, keepdim=True).values.clamp_min(1e-8)
        dev = ((qs - center) / mad).abs()
        w = torch.where(dev < 1.5, torch.ones_like(dev), 1.5 / dev.clamp_min(1.5))
        return (qs * w).sum(-1) / w.sum(-1).clamp_min(1e-8)
    # tail_aware
    lo_i = max(0, int(round(K * 0.01)))
    hi_i = min(K - 1, int(round(K * 0.99)) - 1)
    q_lo, q_mid, q_hi = qf[:, lo_i], qf[:, K // 2], qf[:, hi_i]
    left, right = q_mid - q_lo, q_hi - q_mid
    spread = (q_hi - q_lo).abs()
    thresh = spread.median() * 1.5 if q.shape[0] > 1 else spread.new_tensor(-1.0)
    left_heavy = (left.abs() > 3.0 * right.abs().clamp_min(1e-8)) & (spread > thresh)
    right_heavy = (right.abs() > 3.0 * left.abs().clamp_min(1e-8)) & (spread > thresh)
    out = _fast_mean(q, tau)
    out = torch.where(left_heavy, q_lo, out)
    return torch.where(right_heavy, q_hi, out)


def interpolate_levels(q_sorted: torch.Tensor, tau: torch.Tensor, levels) -> torch.Tensor:
    """Quantiles at arbitrary ``levels`` from a sorted bank by linear interpolation in tau
    (clamped to the outer quantiles), ``[N, L]``."""
    t = tau.float().to(q_sorted.device)
    lv = torch.as_tensor(levels, dtype=torch.float32, device=q_sorted.device).reshape(-1)
    idx = torch.searchsorted(t, lv, right=True).clamp(1, t.numel() - 1)
    lo, hi = idx - 1, idx
    w = ((lv - t[lo]) / (t[hi] - t[lo])).clamp(0, 1)
    out = q_sorted[:, lo] + w * (q_sorted[:, hi] - q_sorted[:, lo])
    out = torch.where(lv <= t[0], q_sorted[:, :1].expand_as(out), out)
    return torch.where(lv >= t[-1], q_sorted[:, -1:].expand_as(out), out)


def bar_decode(logits: torch.Tensor, borders: torch.Tensor, estimator: str = "mean",
               temperature: float = 1.0) -> torch.Tensor:
    """Point estimate from bar-distribution logits ``[N, nb]`` over bins with edges
    ``borders [nb+1]`` (reference ``predictor.py:948-992``)."""
    if estimator not in BAR_ESTIMATORS:
        raise ValueError(f"unknown bar_point_estimator {estimator!r}; expected one of {BAR_ESTIMATORS}")
    if borders.numel() != logits.shape[-1] + 1:
        raise ValueError("borders must have one more entry than there are bins")
    b = borders.to(device=logits.device, dtype=torch.float32)
    centers = 0.5 * (b[:-1] + b[1:])
    t = temperature if temperature > 0 else 1.0
    p = torch.softmax(logits.float() / t, dim=-1)
    if estimator == "mode":
        return centers[p.argmax(-1)]
    if estimator == "median":
        return centers[(p.cumsum(-1) >= 0.5).int().argmax(-1)]
    return (p * centers).sum(-1)


def uniform_borders(num_bars: int, lo: float = -10.0, hi: float = 10.0) -> torch.Tensor:
    return torch.linspace(lo, hi, num_bars + 1)
