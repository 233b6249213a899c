"""Per-step table shapes for pretraining.

Every step draws one (rows, features, context ratio) shared by all tables and ranks
(from a generator seeded identically on every rank).  Behaviour of the reference
(``training/trainer.py:233-380``):

* rows and features are drawn log-uniformly with a bias toward the maximum
  (``u ** (1 / bias)`` on the unit interval, ``bias = 1`` is plain log-uniform);
* features are rounded up to a multiple of the features-per-group;
* a draw over the element budget (rows x features) is projected onto the budget: the
  feature count is cut to ``budget // rows`` (rounded to the group size), or, if that
  leaves less than one group, the row count is cut instead;
* the result snaps down to the largest bucket of a fixed grid (rows and features) at or
  below the draw, and the context ratio to the nearest allowed ratio bucket;
* an explicit palette of (rows, features, weight) entries, and a palette of context
  ratios, replace the random draws.

Buckets bound the set of distinct shapes a run sees, which keeps memory planning and
any shape-specialised state bounded (the native kernels themselves take any shape).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

SAMPLE_BUCKETS = (64, 128, 256, 512, 768, 1024, 1536, 2048, 3072, 4096, 6144, 8192, 12288, 16384, 24576, 32768,
                  49152)
FEATURE_BUCKETS = (4, 8, 16, 32, 48, 64, 96, 128, 192, 256, 320, 384, 512, 768, 1024)
CONTEXT_RATIO_BUCKETS = (0.30, 0.40, 0.50, 0.60, 0.70, 0.80)


@dataclass
class ShapeConfig:
    min_samples: int = 256
    max_samples: int = 2048
    min_features: int = 2
    max_features: int = 100
    features_per_group: int = 2
    max_budget: int = 250_000
    dim_bias_samples: float = 1.0
    dim_bias_features: float = 1.0
    context_ratio_min: float = 0.5
    context_ratio_max: float = 0.9
    bucketed: bool = True
    shape_palette: list = field(default_factory=list)  # [(rows, features, weight)]
    context_ratio_palette: list = field(default_factory=list)
    fixed: tuple | None = None  # (rows, features)


def shape_support(cfg: ShapeConfig) -> dict:
    """The bucketed (rows, features) pairs reachable under the budget."""
    if cfg.shape_palette:
        shapes = [(int(r), int(f)) for r, f, _w in cfg.shape_palette if int(r) * int(f) <= cfg.max_budget]
    else:
        rows = [r for r in SAMPLE_BUCKETS if cfg.min_samples <= r <= cfg.max_samples]
        feats = [f for f in FEATURE_BUCKETS if cfg.min_features <= f <= cfg.max_features
                 and f % cfg.features_per_group == 0]
        shapes = [(r, f) for r in rows for f in feats if r * f <= cfg.max_budget]
    if not shapes:
        raise ValueError(f"no bucketed shape within rows {cfg.min_samples}..{cfg.max_samples}, features "
                         f"{cfg.min_features}..{cfg.max_features} and budget {cfg.max_budget}")
    rs = sorted({r for r, _ in shapes})
    fs = sorted({f for _, f in shapes})
    return {"shapes": shapes, "sample_buckets": rs, "feature_buckets": fs}


class ShapeSampler:
    def __init__(self, cfg: ShapeConfig, seed: int):
        self.cfg = cfg
        self.rng = np.random.default_rng(seed)  # identical on every rank
        self.support = shape_support(cfg) if cfg.bucketed else None

    def state(self):
        return self.rng.bit_generator.state

    def set_state(self, st):
        self.rng.bit_generator.state = st

    def _log_biased(self, lo: int, hi: int, bias: float) -> int:
        u = self.rng.uniform(0, 1) ** (1.0 / bias)
        return int(np.exp(np.log(lo) + u * (np.log(hi) - np.log(lo))))

    def sample(self) -> tuple[int, int, float]:
        """(rows, features, context ratio)."""
        c, rng = self.cfg, self.rng
        fpg = c.features_per_group
        palette = bool(c.shape_palette)
        if palette:
            w = np.asarray([e[2] for e in c.shape_palette], dtype=np.float64)
            i = int(rng.choice(len(c.shape_palette), p=w / w.sum()))
            n, f = int(c.shape_palette[i][0]), int(c.shape_palette[i][1])
            if n * f > c.max_budget:
                raise ValueError(f"palette shape {n}x{f} exceeds the element budget {c.max_budget}")
        elif c.fixed is not None:
            rng.uniform(0, 1)
            rng.uniform(0, 1)  # keep the stream aligned with the random-shape path
            n, f = int(c.fixed[0]), int(c.fixed[1])
        else:
            n = self._log_biased(c.min_samples, c.max_samples, c.dim_bias_samples)
            f = self._log_biased(c.min_features, c.max_features, c.dim_bias_features)
            f = max(fpg, -(-f // fpg) * fpg)
            if n * f > c.max_budget:  # project onto the budget frontier
                mf = c.max_budget // n
                mf -= mf % fpg
                if mf >= fpg:
                    f = min(f, mf)
                else:
                    f = fpg
                    n = max(c.min_samples, c.max_budget // f)
            if self.support is not None:
                rs = [r for r in self.support["sample_buckets"] if r <= n]
                fs = [x for x in self.support["feature_buckets"] if x <= f]
                n = max(rs) if rs else self.support["sample_buckets"][0]
                f = max(fs) if fs else self.support["feature_buckets"][0]
        if c.context_ratio_palette:
            ratio = float(c.context_ratio_palette[int(rng.integers(len(c.context_ratio_palette)))])
        else:
            ratio = float(rng.uniform(c.context_ratio_min, c.context_ratio_max))
            if c.bucketed:
                ok = [r for r in CONTEXT_RATIO_BUCKETS if c.context_ratio_min <= r <= c.context_ratio_max]
                if ok:
                    ratio = min(ok, key=lambda r: abs(r - ratio))
        return n, f, ratio

    @staticmethod
    def eval_pos(rows: int, ratio: float) -> int:
        return min(max(1, int(rows * ratio)), rows - 1)
