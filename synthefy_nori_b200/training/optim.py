"""Flat-buffer AdamW + EMA on the fused ``adamw_ema`` kernel.

All trainable parameters become views into one fp32 buffer and their ``.grad`` views
into one fp32 gradient buffer, so the optimizer step is two launches (gradient norm
for the clip, then AdamW + EMA in one pass) regardless of the parameter count, and
the data-parallel gradient reduction works on one contiguous buffer.

Semantics match ``torch.optim.AdamW`` (decoupled weight decay, bias correction) after
``clip_grad_norm_(max_norm)`` and the reference EMA ``ema = d * ema + (1 - d) * p``
(reference ``training/trainer.py:38-63, 1544-1552``).
"""

from __future__ import annotations

import numpy as np
import torch


class FlatParams:
    """Re-home a module's trainable parameters into one contiguous fp32 buffer."""

    def __init__(self, params, device, align: int = 64):
        self.params = [p for p in params if p.requires_grad]
        self.offsets = []
        off = 0
        for p in self.params:
            self.offsets.append(off)
            off += (p.numel() + align - 1) // align * align
        self.numel = off
        self.data = torch.zeros(off, device=device, dtype=torch.float32)
        self.grad = torch.zeros(off, device=device, dtype=torch.float32)
        for p, o in zip(self.params, self.offsets):
            n = p.numel()
            self.data[o : o + n].copy_(p.detach().reshape(-1).to(self.data))
            p.data = self.data[o : o + n].view(p.shape)
            p.grad = self.grad[o : o + n].view(p.shape)

    def zero_grad(self) -> None:
        self.grad.zero_()
        for p, o in zip(self.params, self.offsets):
            if p.grad is None or p.grad.data_ptr() != self.grad[o:].data_ptr():
                p.grad = self.grad[o : o + p.numel()].view(p.shape)


class FusedAdamWEMA:
    def __init__(self, flat: FlatParams, lr=1e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, ema_decay=0.999,
                 max_grad_norm=1.0):
        self.flat = flat
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.ema_decay, self.max_grad_norm = ema_decay, max_grad_norm
        self.m = torch.zeros_like(flat.data)
        self.v = torch.zeros_like(flat.data)
        self.ema = flat.data.clone() if ema_decay is not None else None
        self.step_count = 0
        self.norm_sq = torch.zeros(1, device=flat.data.device, dtype=torch.float32)

    def step(self, grad_scale: float = 1.0, skip: torch.Tensor | None = None) -> None:
        """One AdamW + EMA step on the flat buffers. ``grad_scale`` multiplies the
        gradients first (e.g. 1 / world_size after a sum-reduction); ``skip`` (device
        scalar, > 0 = reject the step) is read by the kernel, so no host synchronisation."""
        from synthefy_nori_b200 import ops

        self.step_count += 1
        if not self.flat.data.is_cuda:
            self._step_torch(grad_scale, skip)
            return
        if self.max_grad_norm and self.max_grad_norm > 0:
            self.norm_sq.zero_()
            ops.grad_sumsq(self.flat.grad, self.norm_sq)
        ops.adamw_ema_step(self.flat.data, self.flat.grad, self.m, self.v, lr=self.lr, beta1=self.betas[0],
                           beta2=self.betas[1], eps=self.eps, wd=self.wd, step=self.step_count, ema=self.ema,
                           norm_sq=self.norm_sq if self.max_grad_norm else None,
                           ema_decay=self.ema_decay if self.ema_decay is not None else 0.0,
                           max_norm=self.max_grad_norm or 0.0, grad_scale=grad_scale,
                           skip=None if skip is None else skip.reshape(1).float())

    @torch.no_grad()
    def _step_torch(self, grad_scale, skip) -> None:
        """The same update as plain tensor ops (CPU training, e.g. tests and small fine-tunes)."""
        if skip is not None and float(skip) > 0:
            return
        g = self.flat.grad * grad_scale
        if self.max_grad_norm and self.max_grad_norm > 0:
            norm = float(g.double().norm())
            if not np.isfinite(norm):
                return
            g = g * min(1.0, self.max_grad_norm / (norm + 1e-6))
        b1, b2 = self.betas
        p = self.flat.data
        p.mul_(1.0 - self.lr * self.wd)
        self.m.mul_(b1).add_(g, alpha=1 - b1)
        self.v.mul_(b2).addcmul_(g, g, value=1 - b2)
        denom = (self.v / (1 - b2 ** self.step_count)).sqrt_().add_(self.eps)
        p.addcdiv_(self.m, denom, value=-self.lr / (1 - b1 ** self.step_count))
        if self.ema is not None:
            self.ema.mul_(self.ema_decay).add_(p, alpha=1 - self.ema_decay)

    def ema_state_dict(self, model) -> dict:
        """Model state dict with EMA weights in place of the trainable parameters."""
        sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
        if self.ema is None:
            return sd
        by_ptr = {p.data_ptr(): (o, p) for p, o in zip(self.flat.params, self.flat.offsets)}
        for k, v in model.state_dict().items():
            hit = by_ptr.get(v.data_ptr())
            if hit is not None:
                o, p = hit
                sd[k] = self.ema[o : o + p.numel()].view(p.shape).clone()
        return sd

    def state_dict(self) -> dict:
        return {"m": self.m, "v": self.v, "ema": self.ema, "step": self.step_count, "lr": self.lr}

    def load_state_dict(self, sd: dict) -> None:
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        if self.ema is not None and sd.get("ema") is not None:
            self.ema.copy_(sd["ema"])
        self.step_count = int(sd["step"])
        self.lr = float(sd.get("lr", self.lr))
