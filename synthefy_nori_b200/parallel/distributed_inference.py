"""Data-parallel inference over the ranks of one node.

Parity target: reference ``inference/inference_method.py:48-209`` (query rows strided over
ranks by a non-padding sampler, every rank predicts its rows against the replicated
context, results gathered and re-ordered; enabled by ``inference_with_DDP=True``) and
independent tables spread over the GPUs (table data parallelism).  The reference gathers
pickled CPU objects (``all_gather_object``); here the per-rank outputs stay on the device
and are gathered with one collective of a padded tensor (NVLink on a B200 node), then
un-strided on every rank.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def _world(group=None) -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def strided_rows(n: int, rank: int, world: int) -> torch.Tensor:
    """Rows ``rank, rank + world, ...`` of ``n`` (no padding; the last ranks may get one fewer)."""
    return torch.arange(rank, n, world)


def gather_rows(local: torch.Tensor, n: int, group=None) -> torch.Tensor:
    """Inverse of ``strided_rows``: every rank's ``local [n_r, ...]`` -> ``[n, ...]`` on all ranks."""
    rank, world = _world(group)
    if world == 1:
        return local
    cap = (n + world - 1) // world
    buf = local.new_zeros((cap,) + tuple(local.shape[1:]))
    buf[: local.shape[0]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf.contiguous(), group=group)
    out = local.new_empty((n,) + tuple(local.shape[1:]))
    for r in range(world):
        idx = strided_rows(n, r, world)
        out[idx.to(out.device)] = parts[r][: idx.numel()]
    return out


class DistributedInference:
    """Query-row sharding around a ``NoriPredictor``: ``predict_raw`` on each rank's strided
    rows, gathered in the original order on every rank."""

    def __init__(self, predictor, group=None):
        self.predictor, self.group = predictor, group

    def predict_raw(self, ctx, X) -> torch.Tensor:
        X = torch.as_tensor(X)
        rank, world = _world(self.group)
        idx = strided_rows(X.shape[0], rank, world)
        local = self.predictor.predict_raw(ctx, X[idx]) if idx.numel() else \
            self.predictor.predict_raw(ctx, X[:1])[:0]
        return gather_rows(local, X.shape[0], self.group)


def table_parallel_predict(model, x_ctx: torch.Tensor, y_ctx: torch.Tensor, x_query: torch.Tensor, *,
                           cache_dtype: str = "bf16", group=None) -> torch.Tensor:
    """Independent tables ``[B, ...]`` split contiguously over ranks: each rank builds the
    context caches of its tables and predicts their queries; outputs ``[B, Nq, K]`` are
    gathered on every rank."""
    rank, world = _world(group)
    B = x_ctx.shape[0]
    per = (B + world - 1) // world
    lo, hi = min(rank * per, B), min((rank + 1) * per, B)
    with torch.no_grad():
        if hi > lo:
            cache = model.build_context_cache(x_ctx[lo:hi], y_ctx[lo:hi], cache_dtype=cache_dtype)
            out = model.apply_context_cache(x_query[lo:hi], cache).float()
        else:
            out = None
    if world == 1:
        return out
    K = len(model.regression_quantiles)
    buf = torch.zeros(per, x_query.shape[1], K, device=x_query.device)
    if out is not None:
        buf[: hi - lo] = out
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat(parts, 0)[:B]
