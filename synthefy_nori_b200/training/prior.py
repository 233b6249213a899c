"""Batched synthetic training tables generated on the GPU.

``scm_prior_batch`` (the benchmark's pretraining prior): each table is a random
structural causal model realised as a random MLP - Gaussian root causes, a first linear
projection, then ``L - 1`` layers ``h <- W act(h) + sigma eps`` with weights
``N(0, 1 / fan_in)``, a per-(table, layer) activation drawn from {tanh, relu, sin},
values clamped to +/-100; features and the target are distinct hidden units picked at
random from all layers (so the target is causally related to some features and not
others).  Tables of one batch share their row count (the reference trainer samples one
shape per step); feature counts differ per table and unused feature columns are zero.
Every layer of every table runs in one ``scm_act`` + one ``scm_linear`` launch
(``csrc/prior.cu``), so a step's batch costs ``2 L`` kernel launches whatever its size.

``mixture_prior_batch`` draws from the full prior mixture instead (meta-sampled MLP /
tree SCMs, GP, quadratic, sparse-nonlinear, lookup, categorical-dominant, binary,
temporal and low-dimensional families, with the augmentations), see
``training/scm_prior.py`` and ``training/generators.py``.

A batch is a pure function of its seed.
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


_ACT_CODES = (0, 6, 15)  # tanh, relu, sin in the scm_act activation table


@torch.no_grad()
def scm_prior_batch(cfg: PriorConfig, batch_size: int, n_rows: int, eval_pos: int, seed: int,
                    device: torch.device) -> Batch:
    if device.type != "cuda":
        return _scm_prior_batch_torch(cfg, batch_size, n_rows, eval_pos, seed, device)
    from synthefy_nori_b200 import ops

    C = ops.lib()
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    B, N, Hd, L = batch_size, n_rows, cfg.hidden, cfg.max_layers
    Hp = -(-Hd // 32) * 32
    cg = torch.Generator().manual_seed(int(seed))  # host draws (small per-table integers)
    n_layers = torch.randint(cfg.min_layers, cfg.max_layers + 1, (B,), generator=cg)
    width = torch.randint(max(16, cfg.max_features // 4), Hd + 1, (B,), generator=cg)
    n_root = torch.randint(cfg.root_causes[0], cfg.root_causes[1] + 1, (B,), generator=cg)
    noise = cfg.noise_std[0] + (cfg.noise_std[1] - cfg.noise_std[0]) * torch.rand(B, generator=cg)
    act = torch.tensor(_ACT_CODES, dtype=torch.int32)[torch.randint(0, 3, (B, L), generator=cg)]
    n_feat = torch.randint(cfg.min_features, cfg.max_features + 1, (B,), generator=cg)
    Rp = -(-cfg.root_causes[1] // 4) * 4
    cols = torch.arange(Hp, device=device)
    roots = torch.randn(B, N, Rp, generator=g, device=device) * (
        torch.arange(Rp, device=device).view(1, 1, -1) < n_root.to(device).view(-1, 1, 1)).float()
    wmask = (cols.view(1, -1) < width.to(device).view(-1, 1)).float()  # [B, Hp]
    units = []
    h = roots
    zeros_b = torch.zeros(B, Hp, device=device)
    ones = torch.ones(B, device=device)
    ident_mean, ident_rstd = torch.zeros(B, Hp, device=device), torch.ones(B, Hp, device=device)
    rff = torch.zeros(B, 3, 256, device=device)
    for layer in range(L):
        live = (layer < n_layers).to(torch.int32)
        out_w = (width * live).to(torch.int32).to(device)
        if layer == 0:
            A = h
            fan_in = n_root.float().to(device).view(B, 1, 1)
            sig = zeros_b
        else:
            A = C.scm_act(h, act[:, layer].contiguous().to(device), ones, torch.zeros(B, device=device),
                          (width * live).to(torch.int32).to(device), ident_mean, ident_rstd, rff)
            fan_in = width.float().to(device).view(B, 1, 1)
            sig = (noise.to(device).view(B, 1) * wmask).contiguous()
        k_in = A.shape[-1]
        kmask = wmask if layer > 0 else (torch.arange(Rp, device=device).view(1, -1) < n_root.to(device).view(-1, 1)
                                         ).float()
        W = torch.randn(B, Hp, k_in, generator=g, device=device) / fan_in.sqrt()
        W = W * wmask.unsqueeze(2) * kmask.unsqueeze(1)
        csum = torch.zeros(B, Hp, device=device, dtype=torch.float64)
        csq = torch.zeros_like(csum)
        h = C.scm_linear(A.contiguous(), W.contiguous(), zeros_b, sig, out_w, eval_pos,
                         (int(seed) * 1000003 + layer) & 0x3FFFFFFFFFFFFFFF, layer, csum, csq)
        units.append(h)
    return _select(cfg, units, n_layers, width, n_feat, B, N, Hp, eval_pos, g, device)


def _select(cfg, units, n_layers, width, n_feat, B, N, Hp, eval_pos, g, device):
    L = len(units)
    allu = torch.cat(units, -1)  # [B, N, L*Hp]
    idx = torch.arange(L * Hp, device=device).view(1, -1)
    valid = (idx % Hp < width.to(device).view(-1, 1)) & (idx // Hp < n_layers.to(device).view(-1, 1))
    score = torch.rand(B, L * Hp, generator=g, device=device) + (~valid).float() * 2.0
    order = score.argsort(-1)
    Fp = cfg.pad_features
    pick = order[:, : Fp + 1]
    sel = torch.gather(allu, 2, pick.view(B, 1, -1).expand(B, N, Fp + 1))
    y = sel[:, :, Fp]
    x = sel[:, :, :Fp] * (torch.arange(Fp, device=device).view(1, 1, -1) < n_feat.to(device).view(-1, 1, 1)).float()
    mu = y[:, :eval_pos].mean(1, keepdim=True)
    sd = y[:, :eval_pos].std(1, keepdim=True).clamp_min(1e-6)
    y = (y - mu) / sd
    return Batch(x=x.contiguous(), y=y.contiguous(), eval_pos=int(eval_pos), n_features=n_feat.to(device))


@torch.no_grad()
def _scm_prior_batch_torch(cfg: PriorConfig, batch_size: int, n_rows: int, eval_pos: int, seed: int,
                           device: torch.device) -> Batch:
    """The same prior as plain tensor ops (CPU callers and the kernel's oracle)."""
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    B, N, Hd, L = batch_size, n_rows, cfg.hidden, cfg.max_layers
    Hp = -(-Hd // 32) * 32
    cg = torch.Generator().manual_seed(int(seed))
    n_layers = torch.randint(cfg.min_layers, cfg.max_layers + 1, (B,), generator=cg)
    width = torch.randint(max(16, cfg.max_features // 4), Hd + 1, (B,), generator=cg)
    n_root = torch.randint(cfg.root_causes[0], cfg.root_causes[1] + 1, (B,), generator=cg)
    noise = cfg.noise_std[0] + (cfg.noise_std[1] - cfg.noise_std[0]) * torch.rand(B, generator=cg)
    act = torch.tensor(_ACT_CODES)[torch.randint(0, 3, (B, L), generator=cg)]
    n_feat = torch.randint(cfg.min_features, cfg.max_features + 1, (B,), generator=cg)
    Rp = -(-cfg.root_causes[1] // 4) * 4
    wmask = (torch.arange(Hp).view(1, -1) < width.view(-1, 1)).float().to(device)
    rmask = (torch.arange(Rp).view(1, -1) < n_root.view(-1, 1)).float().to(device)
    h = torch.randn(B, N, Rp, generator=g, device=device) * rmask.unsqueeze(1)
    units = []
    for layer in range(L):
        live = (layer < n_layers).view(B, 1, 1).to(device)
        if layer == 0:
            A, fan_in, kmask, sig = h, n_root.float(), rmask, torch.zeros(B, 1, 1, device=device)
        else:
            a = act[:, layer].view(B, 1, 1).to(device)
            A = torch.where(a == 0, torch.tanh(h), torch.where(a == 6, torch.relu(h), torch.sin(h))) * wmask.unsqueeze(1)
            fan_in, kmask, sig = width.float(), wmask, noise.view(B, 1, 1).to(device)
        W = torch.randn(B, Hp, A.shape[-1], generator=g, device=device) / fan_in.to(device).view(B, 1, 1).sqrt()
        W = W * wmask.unsqueeze(2) * kmask.unsqueeze(1)
        z = torch.bmm(A, W.transpose(1, 2)) + sig * torch.randn(B, N, Hp, generator=g, device=device)
        h = torch.where(live, z.clamp(-100, 100) * wmask.unsqueeze(1), torch.zeros_like(z))
        units.append(h)
    return _select(cfg, units, n_layers, width, n_feat, B, N, Hp, eval_pos, g, device)


def mixture_prior_batch(batch_size: int, n_rows: int, eval_pos: int, seed: int, device: torch.device,
                        min_features: int = 5, max_features: int = 100, pad_features: int = 100,
                        family_probs: dict | None = None, augment: bool = True) -> Batch:
    """A batch from the full prior mixture (see ``training/generators.py``)."""
    from synthefy_nori_b200.training.generators import generate_batch

    x, y, n_feat, _ = generate_batch(batch_size, n_rows, eval_pos, seed, device, min_features=min_features,
                                     max_features=max_features, pad_features=pad_features, family_probs=family_probs,
                                     augment=augment)
    return Batch(x=x, y=y, eval_pos=int(eval_pos), n_features=n_feat)
