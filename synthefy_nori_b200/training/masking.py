"""Query-row feature masks for masked-cell training (reference ``training/masking.py:14-96``).

Three patterns, drawn per episode: ``cell`` (each cell independently with probability
``ratio``), ``column`` (``round(ratio * F)`` whole columns, at least one), ``block`` (up
to ten random rectangles until about ``ratio`` of the cells are covered).  Masks are
built on the device with a seeded ``torch.Generator`` for the whole batch at once.
"""

from __future__ import annotations

import torch

MASK_TYPES = ("cell", "column", "block")


def create_masks(n_query: int, n_features: int, ratio: float, kind: str, generator: torch.Generator | None = None,
                 device=None) -> torch.Tensor:
    """Bool mask ``[n_query, n_features]``, True where masked."""
    dev = torch.device("cpu") if device is None else torch.device(device)
    g = generator
    if kind == "cell":
        return (torch.rand(n_query, n_features, generator=g) < ratio).to(dev)
    if kind == "column":
        k = max(1, int(round(n_features * ratio)))
        cols = torch.randperm(n_features, generator=g)[:k]
        m = torch.zeros(n_query, n_features, dtype=torch.bool)
        m[:, cols] = True
        return m.to(dev)
    if kind == "block":
        target = int(round(n_query * n_features * ratio))
        m = torch.zeros(n_query, n_features, dtype=torch.bool)
        for _ in range(10):
            have = int(m.sum())
            if have >= target:
                break
            rows = int(torch.randint(1, n_query + 1, (1,), generator=g))
            cols = max(1, min((target - have) // rows, n_features))
            r0 = int(torch.randint(0, max(1, n_query - rows + 1), (1,), generator=g))
            c0 = int(torch.randint(0, max(1, n_features - cols + 1), (1,), generator=g))
            m[r0 : r0 + rows, c0 : c0 + cols] = True
        return m.to(dev)
    raise ValueError(f"unknown mask type {kind!r}; expected one of {MASK_TYPES}")


def batch_masks(batch: int, n_query: int, n_features: int, *, min_ratio: float = 0.1, max_ratio: float = 0.4,
                seed: int = 0, device=None) -> torch.Tensor:
    """Per-episode random pattern and ratio, ``[batch, n_query, n_features]``."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(batch):
        kind = MASK_TYPES[int(torch.randint(0, 3, (1,), generator=g))]
        ratio = float(min_ratio + (max_ratio - min_ratio) * torch.rand(1, generator=g))
        out.append(create_masks(n_query, n_features, ratio, kind, g))
    return torch.stack(out).to(device if device is not None else "cpu")


def apply_query_masks(x: torch.Tensor, eval_pos: int, masks: torch.Tensor) -> torch.Tensor:
    """NaN-out masked query cells of ``x [B, N, F]`` (the model's missing-value path then
    embeds them with its mask embedding)."""
    out = x.clone()
    q = out[:, eval_pos:]
    q[masks[:, :, : q.shape[2]].to(q.device)] = float("nan")
    return out
