"""In-context learnability filter for synthetic training tables.

A frozen pretrained model (a Nori checkpoint, or any model with the same forward
contract) predicts every candidate table's query rows from its context rows; a
regression table is kept only if that prediction reaches ``min_r2`` on the queries.
Tables that fail are regenerated (new seeds) for up to ``max_rounds`` rounds; a slot
still failing after that raises instead of training on a rejected table.  Before the
model runs, a numeric health mask rejects tables with non-finite targets, infinite
features, constant context or query targets, or no feature that varies in the context
and is observed in the queries.  Behaviour of the reference
(``training/trainer.py:507-840``, ``training/filtering.py``).

B200 design: the candidates are already on the device; the whole batch is scored by
one forward of the frozen model (bf16, the native kernels when the model supports
them), the point prediction is the quantile-distribution mean, and only the boolean
mask comes back to the host.
"""

from __future__ import annotations

import torch


def health_mask(X: torch.Tensor, y: torch.Tensor, n_ctx: int) -> torch.Tensor:
    """[B] bool: tables fit to be scored (see module docstring)."""
    if X.dim() != 3 or y.dim() != 2 or X.shape[:2] != y.shape:
        raise ValueError("health_mask expects X [B, N, F] and y [B, N]")
    if not 0 < n_ctx < X.shape[1]:
        raise ValueError("context rows must be in [1, N - 1]")
    ok = torch.isfinite(y).all(1) & ~torch.isinf(X).flatten(1).any(1)
    yc, yq = y[:, :n_ctx], y[:, n_ctx:]
    ok &= (yc.amax(1) - yc.amin(1)) > 1e-8
    ok &= (yq.amax(1) - yq.amin(1)) > 1e-8
    xc = X[:, :n_ctx]
    fin = torch.isfinite(xc)
    cnt = fin.sum(1)
    mn = torch.where(fin, xc, torch.full_like(xc, float("inf"))).amin(1)
    mx = torch.where(fin, xc, torch.full_like(xc, float("-inf"))).amax(1)
    varying = (cnt >= 2) & torch.isfinite(mn) & torch.isfinite(mx) & ((mx - mn) > 1e-8)
    observed = torch.isfinite(X[:, n_ctx:]).any(1)
    return ok & (varying & observed).any(1)


def regression_mean(model, out: torch.Tensor) -> torch.Tensor:
    """Point prediction from a regression head output [B, Nq, K] in the model's units."""
    K = out.shape[-1]
    head = getattr(model, "regression_loss", "mse" if K == 1 else None)
    if head == "pinball":
        from synthefy_nori_b200.inference.decode import quantile_mean

        taus = torch.as_tensor(model.regression_quantiles, device=out.device, dtype=torch.float32)
        return quantile_mean(out.float(), taus)
    if head == "bar_distribution":
        b = model.bar_borders_buffer.to(out.device, torch.float32)
        return (out.float().softmax(-1) * (b[1:] + b[:-1]) * 0.5).sum(-1)
    if K == 1:
        return out[..., 0].float()
    raise ValueError(f"unsupported regression head {head!r} with {K} outputs")


class _RegeneratingFilter:
    """Accept / regenerate loop shared by the filters: ``score`` gives one number per table
    and a table passes when it is above ``threshold``."""

    threshold = 0.0

    def __init__(self, max_rounds: int):
        self.max_rounds = int(max_rounds)
        self.stats = {"episodes": 0, "first_round_rejects": 0, "rounds_used": 0}

    def score(self, X: torch.Tensor, y: torch.Tensor, n_ctx: int) -> torch.Tensor:  # pragma: no cover - abstract
        raise NotImplementedError

    def filter(self, X, y, n_ctx, regenerate):
        """Replace rejected tables with ``regenerate(slots, round) -> (X_new, y_new)``
        until every slot passes; returns the accepted (X, y)."""
        B = X.shape[0]
        self.stats["episodes"] += B
        passed = self.score(X, y, n_ctx) > self.threshold
        first = int((~passed).sum())
        self.stats["first_round_rejects"] += first
        rnd = 0
        while not bool(passed.all()):
            rnd += 1
            if rnd > self.max_rounds:
                raise RuntimeError(f"{type(self).__name__}: {int((~passed).sum())} table slot(s) still rejected "
                                   f"after {self.max_rounds} regeneration rounds")
            slots = (~passed).nonzero().flatten()
            Xn, yn = regenerate(slots.tolist(), rnd)
            X[slots], y[slots] = Xn, yn
            passed[slots] = self.score(Xn, yn, n_ctx) > self.threshold
        self.stats["rounds_used"] += rnd
        return X, y


class ICLFilter(_RegeneratingFilter):
    def __init__(self, model, device, min_r2: float = 0.05, max_rounds: int = 6):
        super().__init__(max_rounds)
        self.model = model.to(device).eval()
        for p in self.model.parameters():
            p.requires_grad_(False)
        self.device = device
        self.min_r2 = self.threshold = float(min_r2)

    @torch.no_grad()
    def score(self, X: torch.Tensor, y: torch.Tensor, n_ctx: int) -> torch.Tensor:
        """[B] query-row R^2 of the frozen model (-inf for unhealthy tables)."""
        B = X.shape[0]
        r2 = torch.full((B,), float("-inf"), device=X.device)
        ok = health_mask(X, y, n_ctx)
        idx = ok.nonzero().flatten()
        if idx.numel() == 0:
            return r2
        Xs = torch.nan_to_num(X[idx].float(), nan=0.0)
        ys = y[idx].float()
        mu, sd = ys[:, :n_ctx].mean(1, keepdim=True), ys[:, :n_ctx].std(1, unbiased=False, keepdim=True)
        ys = (ys - mu) / sd.clamp(min=1e-8)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=X.is_cuda):
            out = self.model(Xs, ys[:, :n_ctx], eval_pos=n_ctx, task_type="reg")
        out = out["reg_output"] if isinstance(out, dict) else out
        pred = regression_mean(self.model, out[:, : X.shape[1] - n_ctx])
        true = ys[:, n_ctx:]
        ss_res = ((true - pred) ** 2).sum(1)
        ss_tot = ((true - true.mean(1, keepdim=True)) ** 2).sum(1).clamp(min=1e-8)
        r2[idx] = 1.0 - ss_res / ss_tot
        return r2


def _spread(lo: int, n: int, k: int):
    """``min(k, n)`` row indices spread evenly over ``[lo, lo + n)``."""
    import numpy as np

    return lo + np.linspace(0, n - 1, min(k, n)).round().astype(np.int64)


class TreeLearnabilityFilter(_RegeneratingFilter):
    """Model-free learnability gates (reference ``training/data_generator.py:1202-1426``):

    * learnability: a small extremely-randomised tree ensemble (15 trees, depth 6) fitted on
      up to 1000 context rows must reach ``min_score`` R^2 on up to 1000 query rows;
    * context scaling (``scaling=True``): the same model class (10 trees, depth 5) fitted on
      a geometric ladder of context prefixes (from a quarter of the pool to all of it) must end
      above ``min_score`` and gain more than ``min_improvement`` R^2 from the smallest prefix
      to the full one, i.e. more context has to help.

    The trees run on the host (scikit-learn) over the tables' live columns; health failures
    (``health_mask``) score -inf without fitting anything."""

    def __init__(self, min_score: float = 0.10, max_rounds: int = 6, scaling: bool = False,
                 min_improvement: float = 0.03, learnability: bool = True):
        super().__init__(max_rounds)
        self.min_score, self.scaling, self.learnability = float(min_score), bool(scaling), bool(learnability)
        self.min_improvement = float(min_improvement)
        self.threshold = 0.5  # score() returns 1 (keep) or 0 (reject)

    @staticmethod
    def _fit_score(Xf, yf, Xt, yt, trees: int, depth: int) -> float:
        import warnings

        import numpy as np
        from sklearn.ensemble import ExtraTreesRegressor

        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            m = ExtraTreesRegressor(n_estimators=trees, max_depth=depth, random_state=0, n_jobs=1)
            m.fit(Xf, yf)
            s = float(m.score(Xt, yt))
        return s if np.isfinite(s) else 0.0

    def _keep(self, X, y, n_ctx: int) -> bool:
        import numpy as np

        n = X.shape[0]
        if self.learnability:
            ci, qi = _spread(0, n_ctx, 1000), _spread(n_ctx, n - n_ctx, 1000)
            if len(ci) < 2 or len(qi) < 2 or y[ci].std() <= 1e-8 or y[qi].std() <= 1e-8:
                return False
            if self._fit_score(X[ci], y[ci], X[qi], y[qi], 15, 6) <= self.min_score:
                return False
        if self.scaling:
            if n_ctx < 21 or n - n_ctx < 20:
                return False
            rng = np.random.default_rng(1)
            n_pool = min(n_ctx, 800)
            n_test = max(min(n - n_ctx, 1000 - n_pool), min(n - n_ctx, 20))
            pool = rng.permutation(rng.choice(n_ctx, n_pool, replace=False) if n_ctx > n_pool else np.arange(n_ctx))
            test = n_ctx + (rng.choice(n - n_ctx, n_test, replace=False) if n - n_ctx > n_test
                            else np.arange(n - n_ctx))
            lo = max(20, n_pool // 4)
            if n_pool <= lo:
                return False
            sizes = np.unique(np.geomspace(lo, n_pool, 4).astype(int))
            if len(sizes) < 2:
                return False
            scores = [self._fit_score(X[pool[:k]], y[pool[:k]], X[test], y[test], 10, 5) for k in sizes]
            if not (scores[-1] > self.min_score and scores[-1] - scores[0] > self.min_improvement):
                return False
        return True

    @torch.no_grad()
    def score(self, X: torch.Tensor, y: torch.Tensor, n_ctx: int) -> torch.Tensor:
        ok = health_mask(X, y, n_ctx).cpu()
        Xh = torch.nan_to_num(X.float(), nan=0.0).cpu().numpy()
        yh = y.float().cpu().numpy()
        keep = torch.zeros(X.shape[0], device=X.device)
        for b in range(X.shape[0]):
            if bool(ok[b]):
                live = (Xh[b] != 0).any(0)  # padded feature columns are all zero
                keep[b] = float(self._keep(Xh[b][:, live] if live.any() else Xh[b], yh[b], n_ctx))
        return keep
