"""Regression training objectives.

``pinball_objective`` is the reference's pinball objective (``training/loss.py:45-106``
and the pinball branch of ``compute_ccmm_loss``, 363-575): per episode, the mean over
query rows and quantiles of ``max(tau e, (tau - 1) e)`` (optional tail weights), plus
``monotonicity_weight * mean relu(q_i - q_{i+1})^2`` and ``mse_weight *
mean((mean_tau q - y)^2) / clamp(var(y), 0.01)``; the batch loss is the mean over
episodes.  On CUDA the value and the gradient come from one fused kernel
(``pinball_fused``); ``pinball_objective_torch`` is the fp32 oracle.
"""

from __future__ import annotations

import torch


def pinball_objective_torch(pred, target, quantiles, tail_weight=0.0, monotonicity_weight=0.0, mse_weight=0.0):
    """pred [B, Nq, K], target [B, Nq], quantiles [K] -> scalar (fp32 math)."""
    pred = pred.float()
    target = target.float()
    q = torch.as_tensor(quantiles, device=pred.device, dtype=pred.dtype).view(1, 1, -1)
    var = target.var(dim=1, unbiased=False).clamp(min=0.01)
    e = target.unsqueeze(-1) - pred
    loss = torch.maximum(q * e, (q - 1.0) * e)
    if tail_weight > 0:
        loss = loss * (1.0 + tail_weight * (2.0 * (q - 0.5).abs()))
    per_ep = loss.mean(dim=(1, 2))
    if monotonicity_weight > 0 and pred.shape[-1] > 1:
        per_ep = per_ep + monotonicity_weight * torch.relu(pred[..., :-1] - pred[..., 1:]).pow(2).mean(-1).mean(1)
    if mse_weight > 0:
        per_ep = per_ep + mse_weight * ((pred.mean(-1) - target) ** 2).mean(1) / var
    return per_ep.sum() / pred.shape[0]


class _PinballFused(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, target, quantiles, tail_weight, monotonicity_weight, mse_weight):
        from synthefy_nori_b200 import ops

        B, nq, K = pred.shape
        t = target.float()
        inv_var = 1.0 / t.var(dim=1, unbiased=False).clamp(min=0.01)
        loss, grad = ops.pinball_loss_grad(pred.reshape(B * nq, K).contiguous(), t.reshape(-1).contiguous(),
                                           quantiles.float().contiguous(), inv_var.contiguous(), nq, tail_weight,
                                           monotonicity_weight, mse_weight)
        ctx.save_for_backward(grad.view(B, nq, K))
        return loss[0]

    @staticmethod
    def backward(ctx, gout):
        (grad,) = ctx.saved_tensors
        return grad * gout.to(grad.dtype), None, None, None, None, None


def pinball_objective(pred, target, quantiles, tail_weight=0.0, monotonicity_weight=0.0, mse_weight=0.0):
    if pred.is_cuda:
        q = torch.as_tensor(quantiles, device=pred.device, dtype=torch.float32)
        return _PinballFused.apply(pred, target, q, float(tail_weight), float(monotonicity_weight), float(mse_weight))
    return pinball_objective_torch(pred, target, quantiles, tail_weight, monotonicity_weight, mse_weight)
