"""Batched SCM-prior synthetic tables generated on the GPU.

Each table is drawn from a random structural causal model realised as a random MLP
(reference ``training/scm_prior_generator.py:402-600``, ``MLPSCM``): Gaussian root
causes feed ``L`` layers ``h <- act(W h) + sigma * eps`` with weights
``N(0, 1 / fan_in)``, a per-(table, layer) activation drawn from {tanh, relu, sin},
values clamped to +/-100; features and the target are distinct hidden units picked at
random from all layers (so the target is causally related to some features and not
others).  Tables of one batch share their row count (as the reference's trainer
samples one shape per step); feature counts differ per table and the unused feature
columns are zero (constant columns are "invalid" for the model's feature counter).

Everything is generated as a handful of batched tensor ops from one seeded device
generator, so a step's batch is a pure function of its seed.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class PriorConfig:
    min_rows: int = 256
    max_rows: int = 1024
    min_features: int = 5
    max_features: int = 100
    pad_features: int = 100
    min_ctx_frac: float = 0.5
    max_ctx_frac: float = 0.9
    hidden: int = 128
    min_layers: int = 2
    max_layers: int = 4
    noise_std: tuple = (0.01, 0.3)
    root_causes: tuple = (4, 32)


@dataclass
class Batch:
    x: torch.Tensor  # [B, N, F_pad] fp32
    y: torch.Tensor  # [B, N] fp32 (standardised with context statistics)
    eval_pos: int
    n_features: torch.Tensor  # [B] int


def sample_shape(cfg: PriorConfig, rng: torch.Generator) -> tuple[int, int]:
    """(rows, eval_pos) for one step: rows ~ U[min, max], context fraction ~ U[lo, hi]."""
    n = int(torch.randint(cfg.min_rows, cfg.max_rows + 1, (1,), generator=rng).item())
    frac = cfg.min_ctx_frac + (cfg.max_ctx_frac - cfg.min_ctx_frac) * float(torch.rand(1, generator=rng).item())
    ep = min(max(1, int(n * frac)), n - 1)
    return n, ep


@torch.no_grad()
def scm_prior_batch(cfg: PriorConfig, batch_size: int, n_rows: int, eval_pos: int, seed: int,
                    device: torch.device) -> Batch:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    B, N, Hd = batch_size, n_rows, cfg.hidden
    L = cfg.max_layers

    def U(lo, hi, shape):
        return lo + (hi - lo) * torch.rand(shape, generator=g, device=device)

    n_layers = torch.randint(cfg.min_layers, cfg.max_layers + 1, (B,), generator=g, device=device)
    width = torch.randint(max(16, cfg.max_features // 4), Hd + 1, (B,), generator=g, device=device)
    n_root = torch.randint(cfg.root_causes[0], cfg.root_causes[1] + 1, (B,), generator=g, device=device)
    noise = U(cfg.noise_std[0], cfg.noise_std[1], (B, 1, 1))
    act = torch.randint(0, 3, (B, L), generator=g, device=device)
    cols = torch.arange(Hd, device=device)
    wmask = (cols.view(1, -1) < width.view(-1, 1)).float()  # [B, Hd]
    h = torch.randn(B, N, Hd, generator=g, device=device) * (cols.view(1, 1, -1) < n_root.view(-1, 1, 1)).float()
    units = []
    fan_in = n_root.float().view(B, 1, 1)
    for layer in range(L):
        w = torch.randn(B, Hd, Hd, generator=g, device=device) / fan_in.sqrt()
        w = w * wmask.unsqueeze(1) * wmask.unsqueeze(2)
        z = torch.bmm(h, w.transpose(1, 2))
        a = act[:, layer].view(B, 1, 1)
        z = torch.where(a == 0, torch.tanh(z), torch.where(a == 1, torch.relu(z), torch.sin(z)))
        z = z + noise * torch.randn(B, N, Hd, generator=g, device=device)
        z = z.clamp(-100.0, 100.0) * wmask.unsqueeze(1)
        live = (layer < n_layers).view(B, 1, 1)
        h = torch.where(live, z, h)
        units.append(torch.where(live, z, torch.zeros_like(z)))
        fan_in = width.float().view(B, 1, 1)
    allu = torch.cat(units, -1)  # [B, N, L*Hd]
    valid = (torch.arange(L * Hd, device=device).view(1, -1) % Hd < width.view(-1, 1)) & (
        torch.arange(L * Hd, device=device).view(1, -1) // Hd < n_layers.view(-1, 1))
    score = torch.rand(B, L * Hd, generator=g, device=device) + (~valid).float() * 2.0
    order = score.argsort(-1)
    Fp = cfg.pad_features
    n_feat = torch.randint(cfg.min_features, cfg.max_features + 1, (B,), generator=g, device=device)
    pick = order[:, : Fp + 1]
    sel = torch.gather(allu, 2, pick.view(B, 1, -1).expand(B, N, Fp + 1))
    y = sel[:, :, Fp]
    x = sel[:, :, :Fp] * (torch.arange(Fp, device=device).view(1, 1, -1) < n_feat.view(-1, 1, 1)).float()
    # standardise y with context statistics (reference trainer normalises targets per episode)
    mu = y[:, :eval_pos].mean(1, keepdim=True)
    sd = y[:, :eval_pos].std(1, keepdim=True).clamp_min(1e-6)
    y = (y - mu) / sd
    return Batch(x=x.contiguous(), y=y.contiguous(), eval_pos=int(eval_pos), n_features=n_feat)
