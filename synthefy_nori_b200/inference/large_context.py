"""Large-context policies: which rows form the shared context when a table exceeds the
context window, and how several calls are chained.

Parity target: reference ``inference/policies.py`` (``Problem`` 273-626, policies
642-1077, registry and ``"module:fn[k=v]"`` loader 628-640 / 1079-1170) and
``inference/large_context.py:57-279`` (the driver; default threshold 50,000 context rows).
Every policy shares one context across a block of queries, so the context cache built
for it is reused by all of those queries.

Registered policies:

- ``random``: one random window of ``window`` rows.
- ``target_rank[cap=]``: one window chosen at equal-frequency rank midpoints of y.
- ``cluster_route[groups=8]`` / ``cluster_route_g4``: k-means over the query rows (run
  on the device), each training row joins its nearest query centroid, each group gets its
  own window drawn from its region (backfilled with the rows nearest the centroid).
- ``safeboost[nu=0.5]``: residual boosting over disjoint shards where a stage's
  correction is kept only if it does not lower R^2 on the next, still unseen shard.
- ``boost[nu=0.5,patience=3]``: plain residual boosting with early stopping on the
  out-of-fold R^2.
- ``holdout_gate([...])``: scores candidates on a holdout carved from the training rows
  and runs the winner.

A policy is any callable ``(problem, rng) -> predictions [n_test]``; ``register_policy``
adds one under a name, and ``resolve_policy`` also accepts ``"pkg.mod:fn"`` or
``"path/to/file.py:fn"`` specs with ``[k=v,...]`` keyword arguments.
"""

from __future__ import annotations

import importlib
import importlib.util
import os
import warnings
from typing import Callable, Sequence

import numpy as np
import torch

from synthefy_nori_b200.inference.degradation import DegradedPipelineWarning

DEFAULT_LARGE_CONTEXT_THRESHOLD = 50_000
DEFAULT_POLICY = "cluster_route"
MIN_BOOST_SHARDS = 8
Policy = Callable[..., np.ndarray]
_REGISTRY: dict[str, Policy] = {}


class LargeContextPolicyWarning(UserWarning):
    pass


class LargeContextPolicyFallbackWarning(DegradedPipelineWarning, LargeContextPolicyWarning):
    pass


class LargeContextUnsupportedOutputError(ValueError):
    """A shared-pool policy yields point predictions only (no combined distribution)."""


def r2(y, p) -> float:
    y, p = np.asarray(y, np.float64), np.asarray(p, np.float64)
    ss = ((y - y.mean()) ** 2).sum()
    return float("nan") if ss <= 0 else 1.0 - ((y - p) ** 2).sum() / ss


def large_context_applies(n_train: int, policy, threshold: int | None) -> bool:
    return policy is not None and n_train > (DEFAULT_LARGE_CONTEXT_THRESHOLD if threshold is None else threshold)


class Problem:
    """One table: training rows, query rows, the window size and the prediction primitive
    ``predict_fn(X_ctx, y_ctx, X_query) -> point predictions``."""

    def __init__(self, X_train, y_train, X_test, *, window: int, predict_fn, seed: int = 0,
                 max_query_rows_per_call: int = 200_000, train_cache: dict | None = None):
        self.X_train = np.asarray(X_train, np.float32)
        self.y_train = np.asarray(y_train, np.float64)
        self.X_test = np.asarray(X_test, np.float32)
        self.window = int(max(1, min(window, len(self.X_train))))
        self.predict_fn = predict_fn
        self.seed = int(seed)
        self.run_seed = self.seed
        self.max_query_rows_per_call = int(max_query_rows_per_call)
        self.train_cache = {} if train_cache is None else train_cache
        self.calls = 0

    @property
    def n_train(self) -> int:
        return len(self.X_train)

    @property
    def n_test(self) -> int:
        return len(self.X_test)

    def rng(self, offset: int = 0) -> np.random.Generator:
        return np.random.default_rng(self.seed + offset)

    def predict_arrays(self, X_ctx, y_ctx, X_q) -> np.ndarray:
        out = []
        for s in range(0, len(X_q), self.max_query_rows_per_call):
            self.calls += 1
            out.append(np.asarray(self.predict_fn(X_ctx, y_ctx, X_q[s : s + self.max_query_rows_per_call]),
                                  np.float64).reshape(-1))
        return np.concatenate(out) if out else np.empty(0)

    def predict(self, context_idx, query_idx=None, labels=None) -> np.ndarray:
        ci = np.asarray(context_idx)
        y = self.y_train[ci] if labels is None else np.asarray(labels, np.float64)
        Xq = self.X_test if query_idx is None else self.X_test[np.asarray(query_idx)]
        return self.predict_arrays(self.X_train[ci], y, Xq)

    def shards(self, rng: np.random.Generator, count: int | None = None) -> list:
        n = count or max(1, self.n_train // self.window)
        return [np.sort(s) for s in np.array_split(rng.permutation(self.n_train), n)]

    def subproblem(self, train_idx, test_idx) -> "Problem":
        sub = Problem(self.X_train[train_idx], self.y_train[train_idx], self.X_train[test_idx], window=self.window,
                      predict_fn=self.predict_fn, seed=self.seed, max_query_rows_per_call=self.max_query_rows_per_call)
        sub._parent = self
        return sub


def register_policy(name: str):
    def wrap(fn):
        _REGISTRY[name] = fn
        return fn

    return wrap


def registered_policies() -> tuple[str, ...]:
    return tuple(sorted(_REGISTRY))


@register_policy("random")
def random_window(problem: Problem, rng) -> np.ndarray:
    return problem.predict(rng.permutation(problem.n_train)[: problem.window])


@register_policy("target_rank")
def target_rank(problem: Problem, rng, cap: int | None = None) -> np.ndarray:
    cap = problem.window if cap is None else int(cap)
    if cap < 1 or cap > problem.window:
        raise ValueError(f"target_rank cap must lie in [1, window={problem.window}], got {cap}")
    if not np.isfinite(problem.y_train).all():
        raise ValueError("target_rank requires finite context targets")
    if problem.n_train <= cap:
        return problem.predict(np.arange(problem.n_train))
    order = np.argsort(problem.y_train, kind="stable")
    pick = np.floor((np.arange(cap) + 0.5) * problem.n_train / cap).astype(np.int64)
    return problem.predict(np.sort(order[pick]))


def _standardise(train: np.ndarray, test: np.ndarray):
    med = np.nanmedian(train, 0)
    med = np.where(np.isfinite(med), med, 0.0)
    a = np.where(np.isfinite(train), train, med)
    b = np.where(np.isfinite(test), test, med)
    mu, sd = a.mean(0), a.std(0)
    sd = np.where(sd > 0, sd, 1.0)
    return (a - mu) / sd, (b - mu) / sd


def kmeans(points: torch.Tensor, k: int, seed: int, iters: int = 25) -> tuple[torch.Tensor, torch.Tensor]:
    """Lloyd's k-means with k-means++ seeding, on the points' device."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    n = points.shape[0]
    cent = points[torch.randint(n, (1,), generator=g)].clone()
    for _ in range(1, k):
        d2 = torch.cdist(points, cent).min(1).values.pow(2).cpu()
        p = d2 / d2.sum() if float(d2.sum()) > 0 else torch.full((n,), 1.0 / n)
        cent = torch.cat([cent, points[torch.multinomial(p, 1, generator=g).to(points.device)]], 0)
    for _ in range(iters):
        lab = torch.cdist(points, cent).argmin(1)
        s = torch.zeros_like(cent).index_add_(0, lab, points)
        c = torch.bincount(lab, minlength=k).to(points.dtype).unsqueeze(1)
        cent = torch.where(c > 0, s / c.clamp_min(1), cent)
    return torch.cdist(points, cent).argmin(1), cent


@register_policy("cluster_route")
def cluster_route(problem: Problem, rng, groups: int = 8) -> np.ndarray:
    tr, te = _standardise(problem.X_train, problem.X_test)
    dev = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
    groups = max(1, min(int(groups), problem.n_test))
    te_t = torch.as_tensor(te, dtype=torch.float32, device=dev)
    tr_t = torch.as_tensor(tr, dtype=torch.float32, device=dev)
    qlab, cent = kmeans(te_t, groups, problem.seed)
    tlab = torch.cat([torch.cdist(tr_t[s : s + 65536], cent).argmin(1) for s in range(0, len(tr_t), 65536)])
    qlab, tlab = qlab.cpu().numpy(), tlab.cpu().numpy()
    preds = np.zeros(problem.n_test)
    for gi in range(groups):
        q = np.flatnonzero(qlab == gi)
        if not len(q):
            continue
        pool = np.flatnonzero(tlab == gi)
        if len(pool) < problem.window:
            d2 = ((tr_t - cent[gi]) ** 2).sum(1)
            pool = torch.argsort(d2)[: problem.window].cpu().numpy()
        else:
            pool = problem.rng(gi + 1).permutation(pool)[: problem.window]
        preds[q] = problem.predict(np.sort(pool), query_idx=q)
    return preds


@register_policy("cluster_route_g4")
def cluster_route_g4(problem: Problem, rng, groups: int = 4) -> np.ndarray:
    return cluster_route(problem, rng, groups=groups)


def _shards_ok(chain: list, name: str) -> bool:
    if len(chain) < 2:
        warnings.warn(f"{name}: only {len(chain)} shard(s) of `window` rows; falling back to `random`",
                      LargeContextPolicyFallbackWarning, stacklevel=3)
        return False
    if len(chain) < MIN_BOOST_SHARDS:
        warnings.warn(f"{name}: {len(chain)} shards is below the {MIN_BOOST_SHARDS}-shard floor for boosting",
                      LargeContextPolicyWarning, stacklevel=3)
    return True


def _stage(problem: Problem, shard, labels, later):
    Xq = np.vstack([problem.X_test, problem.X_train[later]]) if len(later) else problem.X_test
    h = problem.predict_arrays(problem.X_train[shard], labels, Xq)
    return h[: problem.n_test], h[problem.n_test :]


def replay_chain(problem: Problem, stages) -> np.ndarray:
    out = np.zeros(problem.n_test)
    for shard, labels, w in stages:
        out += w * problem.predict(shard, labels=labels)
    return out


@register_policy("safeboost")
def safeboost(problem: Problem, rng, nu: float = 0.5, shards: int | None = None) -> np.ndarray:
    key = ("safeboost", nu, shards, problem.run_seed)
    if key in problem.train_cache:
        return replay_chain(problem, problem.train_cache[key])
    chain = problem.shards(rng, shards)
    if not _shards_ok(chain, "safeboost"):
        return random_window(problem, rng)
    stages, F_test, F_train = [], np.zeros(problem.n_test), np.zeros(problem.n_train)
    for k in range(len(chain) - 1):
        shard, nxt = chain[k], chain[k + 1]
        later = np.concatenate(chain[k + 1 :])
        labels = problem.y_train[shard] - F_train[shard]
        h_test, h_later = _stage(problem, shard, labels, later)
        w = 1.0 if k == 0 else nu
        cand = F_train.copy()
        cand[later] += w * h_later
        if k == 0 or r2(problem.y_train[nxt], cand[nxt]) >= r2(problem.y_train[nxt], F_train[nxt]) - 1e-4:
            F_train, F_test = cand, F_test + w * h_test
            stages.append((shard, labels, w))
    problem.train_cache[key] = stages
    return F_test


@register_policy("boost")
def boost(problem: Problem, rng, nu: float = 0.5, shards: int | None = None, patience: int = 3) -> np.ndarray:
    key = ("boost", nu, shards, patience, problem.run_seed)
    if key in problem.train_cache:
        return replay_chain(problem, problem.train_cache[key])
    chain = problem.shards(rng, shards)
    if not _shards_ok(chain, "boost"):
        return random_window(problem, rng)
    stages, F_test, F_train = [], np.zeros(problem.n_test), np.zeros(problem.n_train)
    best_test, best_len, best_oof, stale = F_test.copy(), 0, -np.inf, 0
    for k, shard in enumerate(chain):
        labels = problem.y_train[shard] - F_train[shard]
        later = np.concatenate(chain[k + 1 :]) if k + 1 < len(chain) else np.empty(0, np.int64)
        h_test, h_later = _stage(problem, shard, labels, later)
        F_test = F_test + nu * h_test
        stages.append((shard, labels, nu))
        if len(later):
            F_train[later] += nu * h_later
        if k + 1 >= len(chain):
            best_test, best_len = F_test.copy(), len(stages)
            break
        oof = r2(problem.y_train[chain[k + 1]], F_train[chain[k + 1]])
        if oof > best_oof + 1e-4:
            best_oof, best_test, best_len, stale = oof, F_test.copy(), len(stages), 0
        else:
            stale += 1
            if stale >= patience:
                break
    if not best_len:
        warnings.warn("boost: no stage improved out-of-fold R^2; falling back to `random`",
                      LargeContextPolicyFallbackWarning, stacklevel=2)
        return random_window(problem, rng)
    problem.train_cache[key] = stages[:best_len]
    return best_test


def holdout_gate(candidates: Sequence, holdout: int = 2000, strategy: str = "random") -> Policy:
    if strategy not in ("random", "tail"):
        raise ValueError("holdout strategy must be 'random' or 'tail'")
    resolved = [resolve_policy(c) for c in candidates]

    def gate(problem: Problem, rng) -> np.ndarray:
        key = ("gate", tuple(n for n, _ in resolved), holdout, strategy, problem.run_seed)
        winner = problem.train_cache.get(key)
        if winner is None:
            h = min(holdout, max(1, problem.n_train // 5))
            idx = (np.arange(problem.n_train - h, problem.n_train) if strategy == "tail"
                   else np.sort(problem.rng(991).permutation(problem.n_train)[:h]))
            rest = np.setdiff1d(np.arange(problem.n_train), idx)
            sub = problem.subproblem(rest, idx)
            scores = {n: r2(problem.y_train[idx], fn(sub, sub.rng())) for n, fn in resolved}
            problem.calls += sub.calls
            winner = max(scores, key=lambda n: -np.inf if np.isnan(scores[n]) else scores[n])
            problem.train_cache[key] = winner
        gate.last_winner = winner
        return dict(resolved)[winner](problem, rng)

    gate.last_winner = None
    return gate


def _parse_params(text: str) -> dict:
    out = {}
    for part in filter(None, (p.strip() for p in text.split(","))):
        k, _, v = part.partition("=")
        if not _:
            raise ValueError(f"policy parameter {part!r} must be key=value")
        for cast in (int, float):
            try:
                v = cast(v)
                break
            except ValueError:
                continue
        else:
            v = {"true": True, "false": False, "none": None}.get(v.lower(), v)
        out[k.strip()] = v
    return out


def _load(location: str, attr: str):
    if location.endswith(".py") or os.sep in location:
        spec = importlib.util.spec_from_file_location(f"_nori_policy_{abs(hash(location))}", location)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    else:
        mod = importlib.import_module(location)
    return getattr(mod, attr)


def resolve_policy(spec) -> tuple[str, Policy]:
    """``name``, ``name[k=v,...]``, ``module:fn[...]``, ``file.py:fn``, a callable, or a
    list of those (a holdout gate over them)."""
    if callable(spec):
        return getattr(spec, "__name__", "custom"), spec
    if isinstance(spec, (list, tuple)):
        names = [resolve_policy(s)[0] for s in spec]
        return "gate(" + ",".join(names) + ")", holdout_gate(spec)
    if not isinstance(spec, str) or not spec:
        raise TypeError("large_context_policy must be a policy name, spec string, callable or list of those")
    base, params = spec, {}
    if spec.endswith("]") and "[" in spec:
        base, _, rest = spec.partition("[")
        params = _parse_params(rest[:-1])
    if ":" in base:
        loc, _, attr = base.rpartition(":")
        fn = _load(loc, attr)
    elif base in _REGISTRY:
        fn = _REGISTRY[base]
    else:
        raise ValueError(f"unknown large-context policy {base!r}; registered: {registered_policies()}")
    if params:
        inner = fn

        def fn(problem, rng, _inner=inner, _p=params):
            return _inner(problem, rng, **_p)

    return spec, fn


def run_policy(spec, X_train, y_train, X_test, *, window: int, predict_fn, seed: int = 0,
               train_cache: dict | None = None) -> tuple[np.ndarray, dict]:
    """Run a policy; returns (point predictions, report with the call count)."""
    name, fn = resolve_policy(spec)
    prob = Problem(X_train, y_train, X_test, window=window, predict_fn=predict_fn, seed=seed, train_cache=train_cache)
    preds = np.asarray(fn(prob, prob.rng()), np.float64).reshape(-1)
    if preds.shape[0] != prob.n_test:
        raise RuntimeError(f"policy {name!r} returned {preds.shape[0]} predictions for {prob.n_test} queries")
    return preds, {"policy": name, "nori_calls": prob.calls, "window": prob.window,
                   "winner": getattr(fn, "last_winner", None)}
