"""Muon for matrix parameters, AdamW (fused flat-buffer kernel) for the rest.

Parity target: reference ``training/optim.py``: the parameter split (16-56; 2-D
hidden-layer matrices to Muon, embeddings / norms / biases and, unless ``include_nd``,
3-D/4-D attention tensors to AdamW), the Newton-Schulz orthogonalisation (60-85) and
``HybridMuonAdamW`` (180-319).  Muon itself is the published method of K. Jordan et al.
(2024): heavy-ball momentum (Nesterov form) on the gradient, the update replaced by an
approximation of its orthogonal polar factor from five Newton-Schulz iterations with
the quintic coefficients (3.4445, -4.7750, 2.0315) in bf16, then scaled per matrix.

Scaling of the orthogonalised update (``adjust_lr``):
- ``"match_rms_adamw"`` (default, as ``torch.optim.Muon`` in the reference's default
  backend): ``0.2 * sqrt(max(rows, cols))``;
- ``"original"``: ``sqrt(max(1, rows / cols))``;
- ``"nd"``: ``sqrt(max(rows, cols) / min(rows, cols))`` (the reference's ``MuonND``).
Weight decay is decoupled: ``p *= 1 - lr * wd`` before the update.

B200 layout: matrices are grouped by shape and each group is orthogonalised as one
batch (``bmm`` over a stacked ``[G, m, n]`` tensor), so a step costs a handful of
batched GEMMs per distinct shape instead of a chain of small launches per parameter.
The AdamW part runs the fused ``adamw_ema`` kernel on one contiguous tail of the flat
parameter buffer (Muon parameters are laid out first), and the EMA covers the whole
buffer.
"""

from __future__ import annotations

from collections import defaultdict

import torch

from synthefy_nori_b200.training.optim import FlatParams

NS_COEFFS = (3.4445, -4.7750, 2.0315)
_EXCLUDE = ("embedding", "mask_embedding", "y_mask", "feature_positional_embedding")


def split_muon_adamw_params(named_parameters, *, include_embeddings: bool = False, include_nd: bool = False):
    muon, adamw = [], []
    for name, p in named_parameters:
        if not p.requires_grad:
            continue
        is_emb = any(t in name.lower() for t in _EXCLUDE)
        shape_ok = p.ndim == 2 or (include_nd and p.ndim >= 2)
        (muon if shape_ok and (include_embeddings or not is_emb) else adamw).append((name, p))
    return muon, adamw


@torch.no_grad()
def newton_schulz(G: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    """Batched quintic Newton-Schulz on ``G [..., m, n]`` (bf16 inside), returns G's dtype."""
    a, b, c = NS_COEFFS
    X = G.to(torch.bfloat16)
    X = X / (X.flatten(-2).norm(dim=-1)[..., None, None] + eps)
    tall = X.shape[-2] > X.shape[-1]
    if tall:
        X = X.transpose(-2, -1)
    for _ in range(steps):
        A = X @ X.transpose(-2, -1)
        B = b * A + c * (A @ A)
        X = a * X + B @ X
    if tall:
        X = X.transpose(-2, -1)
    return X.to(G.dtype)


def _scale(m: int, n: int, mode: str) -> float:
    if mode == "match_rms_adamw":
        return 0.2 * max(m, n) ** 0.5
    if mode == "original":
        return max(1.0, m / n) ** 0.5
    if mode == "nd":
        return (max(m, n) / min(m, n)) ** 0.5
    raise ValueError(f"unknown adjust_lr {mode!r}")


class HybridMuonAdamW:
    """Muon + fused AdamW + EMA over one flat parameter buffer.

    ``step(grad_scale)`` clips by the global gradient norm (``max_grad_norm``), applies
    Muon to the matrix parameters and AdamW to the rest, then updates the EMA."""

    def __init__(self, model, device, *, lr=3e-4, muon_lr=None, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01,
                 momentum=0.95, nesterov=True, ns_steps=5, adjust_lr="match_rms_adamw", include_embeddings=False,
                 include_nd=False, ema_decay=0.999, max_grad_norm=1.0):
        muon, adamw = split_muon_adamw_params(model.named_parameters(), include_embeddings=include_embeddings,
                                              include_nd=include_nd)
        self.flat = FlatParams([p for _, p in muon] + [p for _, p in adamw], device)
        self.n_muon = len(muon)
        self.split = self.flat.offsets[self.n_muon] if adamw else self.flat.numel
        self.lr, self.muon_lr = lr, muon_lr
        self.betas, self.eps, self.wd = betas, eps, weight_decay
        self.momentum, self.nesterov, self.ns_steps, self.adjust_lr = momentum, nesterov, ns_steps, adjust_lr
        self.ema_decay, self.max_grad_norm = ema_decay, max_grad_norm
        self.m = torch.zeros(self.flat.numel - self.split, device=device)
        self.v = torch.zeros_like(self.m)
        self.ema = self.flat.data.clone() if ema_decay is not None else None
        self.norm_sq = torch.zeros(1, device=device)
        self.step_count = 0
        groups = defaultdict(list)
        for p in self.flat.params[: self.n_muon]:
            groups[(p.numel() // p.shape[-1], p.shape[-1])].append(p)  # N-D: [prod(leading), last]
        # momentum buffers stacked per shape group
        self.groups = [(shape, ps, torch.zeros(len(ps), *shape, device=device)) for shape, ps in groups.items()]

    @torch.no_grad()
    def step(self, grad_scale: float = 1.0, skip: torch.Tensor | None = None) -> None:
        """``skip`` (device scalar, > 0 = reject the step): every update below is blended
        with ``keep = (skip <= 0)`` on the device, so a rejected step changes nothing and
        no host synchronisation is needed."""
        from synthefy_nori_b200 import ops

        self.step_count += 1
        keep = None if skip is None else (skip.reshape(()) <= 0).float()
        grad = self.flat.grad
        if grad_scale != 1.0:
            grad.mul_(grad_scale)
        clip = None
        if self.max_grad_norm and self.max_grad_norm > 0:
            self.norm_sq.zero_()
            if grad.is_cuda and ops.native_available():
                ops.grad_sumsq(grad, self.norm_sq)
            else:
                self.norm_sq.copy_(grad.double().pow(2).sum().float().view(1))
            clip = (self.max_grad_norm / (self.norm_sq.sqrt() + 1e-6)).clamp(max=1.0)
        lr_m = self.muon_lr if self.muon_lr is not None else self.lr
        for (m, n), ps, buf in self.groups:
            g = torch.stack([p.grad.reshape(m, n) for p in ps])
            if clip is not None:
                g.mul_(clip)
            if keep is None:
                buf.mul_(self.momentum).add_(g)
            else:  # buf <- momentum buf + g when kept, unchanged when rejected
                buf.mul_(1.0 - keep * (1.0 - self.momentum)).add_(g * keep)
            eff = g.add(buf, alpha=self.momentum) if self.nesterov else buf
            upd = newton_schulz(eff, self.ns_steps)
            s = _scale(m, n, self.adjust_lr)
            for i, p in enumerate(ps):
                if keep is None:
                    if self.wd:
                        p.mul_(1.0 - lr_m * self.wd)
                    p.add_(upd[i].view_as(p), alpha=-lr_m * s)
                else:
                    if self.wd:
                        p.mul_(1.0 - lr_m * self.wd * keep)
                    p.add_(upd[i].view_as(p) * (-lr_m * s * keep))
        if self.split < self.flat.numel:
            data, g = self.flat.data[self.split :], grad[self.split :]
            if data.is_cuda and ops.native_available():
                ops.adamw_ema_step(data, g, self.m, self.v, lr=self.lr, beta1=self.betas[0], beta2=self.betas[1],
                                   eps=self.eps, wd=self.wd, step=self.step_count, ema=None,
                                   norm_sq=self.norm_sq if clip is not None else None, ema_decay=0.0,
                                   max_norm=self.max_grad_norm or 0.0, grad_scale=1.0,
                                   skip=None if skip is None else skip.reshape(1).float())
            else:
                if keep is not None and float(keep) == 0.0:  # CPU path: a host decision costs nothing
                    pass
                else:
                    self._adamw_torch(data, g * (clip if clip is not None else 1.0))
        if self.ema is not None:
            w = 1.0 - self.ema_decay
            self.ema.lerp_(self.flat.data, w if keep is None else keep * w)

    def _adamw_torch(self, p, g):
        b1, b2 = self.betas
        self.m.mul_(b1).add_(g, alpha=1 - b1)
        self.v.mul_(b2).addcmul_(g, g, value=1 - b2)
        mh = self.m / (1 - b1 ** self.step_count)
        vh = self.v / (1 - b2 ** self.step_count)
        p.mul_(1 - self.lr * self.wd).addcdiv_(mh, vh.sqrt().add_(self.eps), value=-self.lr)

    def zero_grad(self) -> None:
        self.flat.zero_grad()

    def state_dict(self) -> dict:
        return {"m": self.m, "v": self.v, "ema": self.ema, "step": self.step_count,
                "muon_momentum": [b for _, _, b in self.groups]}

    def load_state_dict(self, sd: dict) -> None:
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        if self.ema is not None and sd.get("ema") is not None:
            self.ema.copy_(sd["ema"])
        for (_, _, b), src in zip(self.groups, sd["muon_momentum"]):
            b.copy_(src)
        self.step_count = int(sd["step"])
