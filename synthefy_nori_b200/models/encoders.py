"""Input encoders of the Nori model: column preprocessing, per-cell numeric
embedding, and target (y) embeddings.

Behavioural parity targets (reference paths are relative to the reference
project's ``src/synthefy_nori``):

* context statistics: ``model/encoders.py:12-77`` (finite mean / std, outlier clamp,
  mean-0 std-1 normalisation with the +1e-20 std guard and the +/-100 clip);
* NaN handling: ``model/encoders.py:588-653`` (fill with the finite context mean);
* valid-feature rescale: ``model/encoders.py:656-724`` (per feature group, scale by
  ``sqrt(fpg / n_valid)``);
* scientific-RBF cell embedding: ``model/encoders.py:118-276``;
* mask-embedding encoder + group fusion: ``model/encoders.py:432-585``;
* y encoders: ``model/encoders.py:727-969``.

The module / parameter names are the reference checkpoint's state-dict keys, so a
released ``nori.pt`` loads with ``strict=True``.  The computation here is the plain
PyTorch path; the B200 path replaces the per-cell work with the fused
``feature_embed`` CUDA kernel (``synthefy_nori_b200/csrc/embed.cu``), which is
tested against this module.
"""

from __future__ import annotations

import math
from typing import Any

import torch
import torch.nn as nn


# --------------------------------------------------------------------------------------
# Context statistics (column-wise reductions over context rows)
# --------------------------------------------------------------------------------------


def finite_mean(x: torch.Tensor, dim: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Mean over the finite entries along ``dim`` and the (>=1) finite count."""
    ok = torch.isfinite(x)
    count = ok.sum(dim=dim).clamp(min=1)
    total = torch.where(ok, x, torch.zeros_like(x)).sum(dim=dim)
    return total / count, count


def finite_std(x: torch.Tensor, dim: int, mean: torch.Tensor, count: torch.Tensor) -> torch.Tensor:
    """Unbiased std over the finite entries (denominator ``max(count-1, 1)``)."""
    ok = torch.isfinite(x)
    sq = torch.where(ok, (mean.unsqueeze(dim) - x) ** 2, torch.zeros_like(x))
    return torch.sqrt(sq.sum(dim=dim) / (count - 1).clamp(min=1))


def clamp_outliers(x, sigma, eval_pos, lower=None, upper=None):
    """Two-pass +/- sigma*std outlier bounds from context rows; soft log clamp."""
    if lower is None:
        ctx = x[:, :eval_pos].clone()
        m, c = finite_mean(ctx, 1)
        s = finite_std(ctx, 1, m, c)
        lo, hi = m - sigma * s, m + sigma * s
        ctx[(ctx > hi.unsqueeze(1)) | (ctx < lo.unsqueeze(1))] = float("nan")
        m, c = finite_mean(ctx, 1)
        s = finite_std(ctx, 1, m, c)
        lower, upper = m - sigma * s, m + sigma * s
    x = torch.maximum(-torch.log1p(torch.abs(x)) + lower.unsqueeze(1), x)
    x = torch.minimum(torch.log1p(torch.abs(x)) + upper.unsqueeze(1), x)
    return x, lower, upper


def standardize(x, eval_pos, mean=None, std=None, clip=True):
    """Mean-0 / std-1 with context statistics; std guard 1e-20; clip to +/-100."""
    if mean is None:
        mean, count = finite_mean(x[:, :eval_pos], 1)
        std = finite_std(x[:, :eval_pos], 1, mean, count) + 1e-20
        if x.shape[1] == 1 or eval_pos == 1:
            std = torch.ones_like(std)
    x = (x - mean.unsqueeze(1)) / std.unsqueeze(1)
    if clip:
        x = torch.clamp(x, -100.0, 100.0)
    return x, mean, std


# --------------------------------------------------------------------------------------
# Preprocessing stages (operate on a dict, like the reference pipeline)
# --------------------------------------------------------------------------------------


class NanEncoder(nn.Module):
    """Replace non-finite values by the finite context mean; emit an indicator channel
    (-2 NaN, +2 +inf, +4 -inf).  Honours ``_frozen_nan_mean`` (context-cache path)."""

    def __init__(self, nan_value=-2.0, inf_value=2.0, neg_inf_value=4.0, in_keys=("data",), out_key="nan_encoding"):
        super().__init__()
        self.nan_value, self.inf_value, self.neg_inf_value = nan_value, inf_value, neg_inf_value
        self.in_keys = list(in_keys)
        self.out_key = out_key

    def forward(self, d: dict) -> dict:
        x = d[self.in_keys[0]]
        frozen = d.get("_frozen_nan_mean")
        mean = frozen if frozen is not None else finite_mean(x[:, : d["eval_pos"]], 1)[0]
        d["_nan_mean"] = mean
        is_nan = torch.isnan(x)
        pos_inf = torch.isinf(x) & (x > 0)
        neg_inf = torch.isinf(x) & (x < 0)
        ind = torch.zeros_like(x)
        ind = torch.where(neg_inf, torch.full_like(x, self.neg_inf_value), ind)
        ind = torch.where(pos_inf, torch.full_like(x, self.inf_value), ind)
        ind = torch.where(is_nan, torch.full_like(x, self.nan_value), ind)
        d[self.in_keys[0]] = torch.where(~torch.isfinite(x), mean.unsqueeze(1).expand_as(x), x)
        d[self.out_key] = ind
        return d


class NormalizationEncoder(nn.Module):
    """Context-statistics normalisation (optionally outlier clamp first)."""

    def __init__(self, train_only: bool, normalize_x: bool, remove_outliers: bool, std_sigma: float = 4.0):
        super().__init__()
        self.train_only, self.normalize_x, self.remove_outliers = train_only, normalize_x, remove_outliers
        self.std_sigma = std_sigma

    def forward(self, d: dict) -> dict:
        x = d["data"]
        pos = d["eval_pos"] if self.train_only else x.shape[1]
        frozen = d.get("_frozen_norm_stats")
        cap: dict[str, torch.Tensor] = {}
        if self.remove_outliers:
            lo = frozen.get("lower") if frozen else None
            hi = frozen.get("upper") if frozen else None
            x, lo, hi = clamp_outliers(x, self.std_sigma, pos, lo, hi)
            cap["lower"], cap["upper"] = lo, hi
        if self.normalize_x:
            mean = frozen.get("mean") if frozen else None
            std = frozen.get("std") if frozen else None
            x, mean, std = standardize(x, pos, mean, std)
            d["_norm_mean"], d["_norm_std"] = mean, std
            cap["mean"], cap["std"] = mean, std
        d["data"] = x
        d["_norm_stats"] = cap
        return d


class ValidFeatureEncoder(nn.Module):
    """Count per feature group the context columns that are non-constant (more than one
    finite value and min != max) and rescale the group by ``sqrt(fpg / count)``."""

    def __init__(self, num_features: int, nan_normalize: bool = True, sqrt_normalize: bool = True):
        super().__init__()
        self.num_features, self.nan_normalize, self.sqrt_normalize = num_features, nan_normalize, sqrt_normalize

    def forward(self, d: dict) -> dict:
        x = d["data"]
        frozen = d.get("_frozen_valid_feature_num")
        if frozen is None:
            ctx = x[:, : int(d["eval_pos"])]
            m = d.get("mask")
            if isinstance(m, torch.Tensor) and m.shape == x.shape:
                ctx = torch.where(m[:, : ctx.shape[1]].bool(), torch.full_like(ctx, float("nan")), ctx)
            ok = torch.isfinite(ctx)
            cnt = ok.sum(1)
            mn = torch.where(ok, ctx, torch.full_like(ctx, float("inf"))).amin(1)
            mx = torch.where(ok, ctx, torch.full_like(ctx, float("-inf"))).amax(1)
            valid = (cnt > 1) & (mn != mx)
            nvalid = valid.sum(-1, keepdim=True).clamp(min=1)
        else:
            nvalid = frozen
        d["_valid_feature_num"] = nvalid
        if self.nan_normalize:
            if self.sqrt_normalize:
                x = x * torch.sqrt(self.num_features / nvalid).unsqueeze(1)
            else:
                x = x * (self.num_features / nvalid).unsqueeze(1)
        if x.shape[-1] < self.num_features:
            pad = x.new_zeros(*x.shape[:-1], self.num_features - x.shape[-1])
            x = torch.cat([x, pad], -1)
        d["data"] = x
        return d


class PromptQuantilePLE(nn.Module):
    """Context-only quantile edges per (group, feature) for piecewise-linear encoding
    (Model v3 tokenizer; reference ``model/encoders.py:309-429``)."""

    reference_key = "_prompt_quantile_ple_reference"
    frozen_reference_key = "_frozen_prompt_quantile_ple_reference"

    def __init__(self, n_bins: int):
        super().__init__()
        if n_bins < 2:
            raise ValueError("prompt-quantile PLE requires at least 2 bins")
        self.n_bins = int(n_bins)
        self.register_buffer("quantile_levels", torch.linspace(0.0, 1.0, self.n_bins + 1), persistent=False)

    def forward(self, d: dict) -> dict:
        x, mask = d["data"], d["mask"]
        frozen = d.get(self.frozen_reference_key)
        if frozen is None:
            ep = int(d["eval_pos"])
            valid = torch.isfinite(x) & ~mask.bool()
            ctx, cvalid = x[:, :ep], valid[:, :ep]
            srt = torch.where(cvalid, ctx, torch.full_like(ctx, float("inf"))).permute(0, 2, 3, 1).sort(-1).values
            n = cvalid.sum(1)
            pos = (n - 1).clamp(min=0).to(x.dtype).unsqueeze(-1) * self.quantile_levels.to(x)
            lo_i, hi_i = pos.floor().long(), pos.ceil().long()
            lo, hi = torch.gather(srt, -1, lo_i), torch.gather(srt, -1, hi_i)
            edges = lo + (pos - lo_i.to(pos.dtype)) * (hi - lo)
            edges = torch.where(n.unsqueeze(-1) > 0, edges, torch.zeros_like(edges))
            ref = {"edges": edges.detach()}
        else:
            ref = frozen
        d[self.reference_key] = {"edges": ref["edges"].to(device=x.device, dtype=x.dtype)}
        return d

    @staticmethod
    def encode(x: torch.Tensor, reference: dict) -> torch.Tensor:
        edges = reference["edges"].to(device=x.device, dtype=x.dtype)
        left, right = edges[..., :-1], edges[..., 1:]
        width = right - left
        nz = width > 0
        safe = torch.where(nz, width, torch.ones_like(width))
        v = x.permute(0, 2, 3, 1).unsqueeze(-1)
        c = ((v - left.unsqueeze(-2)) / safe.unsqueeze(-2)).clamp(0.0, 1.0)
        c = torch.where(torch.isfinite(v) & nz.unsqueeze(-2), c, torch.zeros_like(c))
        return c.permute(0, 3, 1, 2, 4).contiguous()


def build_x_preprocess(
    *,
    num_features: int,
    nan_handling_enabled: bool,
    normalize_on_train_only: bool,
    normalize_x: bool,
    remove_outliers: bool,
    normalize_by_used_features: bool,
    prompt_quantile_ple_bins: int = 0,
) -> nn.Sequential:
    """The x preprocessing pipeline (reference ``model/encoders.py:972-1009``)."""
    steps: list[nn.Module] = []
    if nan_handling_enabled:
        steps.append(NanEncoder())
    steps.append(NormalizationEncoder(normalize_on_train_only, normalize_x, remove_outliers))
    steps.append(ValidFeatureEncoder(num_features, nan_normalize=normalize_by_used_features))
    if prompt_quantile_ple_bins:
        steps.append(PromptQuantilePLE(prompt_quantile_ple_bins))
    return nn.Sequential(*steps)


# --------------------------------------------------------------------------------------
# Per-cell numeric embeddings
# --------------------------------------------------------------------------------------


def scientific_decompose(x: torch.Tensor, max_exp: int):
    """|x| = m * 10**e with e = clamp(floor(log10|x|), -max_exp, max_exp); m = 0 for x == 0.

    The reference evaluates this in float64 (``model/encoders.py:218-233``)."""
    a = torch.abs(x)
    zero = a == 0
    safe = torch.where(zero, torch.ones_like(a), a)
    e = torch.clamp(torch.floor(torch.log10(safe)), -max_exp, max_exp).to(torch.int64)
    m = a / (10.0 ** e.to(x.dtype))
    return torch.where(zero, torch.zeros_like(m), m), e


class RBFembedding(nn.Module):
    """Scientific-notation RBF cell embedding.

    Per scalar: mantissa m and decimal exponent e; ``n_kernels`` Gaussian kernels on
    centres ``linspace(0, 10)`` evaluated at m; a gate MLP on the (sign, exponent sign,
    exponent digit) token embeddings gives (gamma, beta) so ``rbf*sigmoid(g)+tanh(b)``;
    LayerNorm; Linear to the embedding width.  ``exp_digit`` only takes 10 values and the
    signs 2 each, so the gate depends on at most 40 distinct control tokens - the fused
    CUDA kernel evaluates the gate MLP once per token instead of once per cell.
    """

    def __init__(
        self,
        embedding_size: int = 96,
        exponent_digits: int = 1,
        token_embed_dim: int = 32,
        n_kernels: int = 32,
        sigma: float = 1.05,
        use_learn_sigma: bool = False,
        center_range=(0.0, 10.0),
        use_learn_embeddings: bool = False,
        as_tokenizer: bool = False,
        use_original_features: bool = False,
        dtype: torch.dtype = torch.float32,
    ):
        super().__init__()
        self.dtype = dtype
        self.n_kernels = n_kernels
        self.exponent_digits = exponent_digits
        self.as_tokenizer = as_tokenizer
        self.use_original_features = use_original_features
        lo, hi = center_range
        centers = (
            torch.tensor([(lo + hi) / 2.0]) if n_kernels <= 1 else torch.linspace(lo, hi, n_kernels, dtype=torch.float32)
        )
        self.register_buffer("centers", centers, persistent=False)
        if use_learn_sigma:
            self.sigma = nn.Parameter(torch.tensor(sigma, dtype=dtype))
        else:
            self.register_buffer("sigma", torch.tensor(sigma, dtype=dtype))
        if exponent_digits > 0:
            self.sign_embedding = nn.Embedding(2, token_embed_dim, dtype=dtype)
            self.exp_sign_embedding = nn.Embedding(2, token_embed_dim, dtype=dtype)
            self.exp_digit_embedding = nn.Embedding(10, token_embed_dim, dtype=dtype)
            if not use_learn_embeddings:
                for emb in (self.sign_embedding, self.exp_sign_embedding, self.exp_digit_embedding):
                    emb.weight.requires_grad = False
            ctrl = (exponent_digits + 2) * token_embed_dim
            self.gate_mlp = nn.Sequential(
                nn.Linear(ctrl, 4 * token_embed_dim, dtype=dtype),
                nn.GELU(),
                nn.Linear(4 * token_embed_dim, 2 * n_kernels, dtype=dtype),
            )
        else:
            self.sign_embedding = self.exp_sign_embedding = self.exp_digit_embedding = None
            self.gate_mlp = None
        self.norm = nn.LayerNorm(n_kernels, dtype=dtype)
        self.out_layer = nn.Linear(n_kernels + (1 if use_original_features else 0), embedding_size, dtype=dtype)

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        # Some checkpoints persisted the (deterministic) centre grid; accept it only if
        # it is exactly the canonical grid.
        key = prefix + "centers"
        c = state_dict.get(key)
        if torch.is_tensor(c) and c.shape == self.centers.shape and torch.equal(c.to(self.centers), self.centers):
            state_dict = dict(state_dict)
            state_dict.pop(key)
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)

    @property
    def max_exp(self) -> int:
        return 10 ** self.exponent_digits - 1

    def control_table(self) -> tuple[torch.Tensor, torch.Tensor]:
        """(gamma, beta) for every (sign, exponent) control token.

        Token index = sign * (2*max_exp+1) + (e + max_exp); returns two
        ``[2*(2*max_exp+1), n_kernels]`` tensors (sigmoid / tanh applied)."""
        me = self.max_exp
        e = torch.arange(-me, me + 1, device=self.sign_embedding.weight.device)
        sign = torch.arange(2, device=e.device)
        sign_i = sign.repeat_interleave(e.numel())
        e_i = e.repeat(2)
        parts = [self.sign_embedding(sign_i), self.exp_sign_embedding((e_i < 0).long())]
        ae = e_i.abs()
        digits = [self.exp_digit_embedding((ae // (10 ** p)) % 10) for p in range(self.exponent_digits)]
        ctrl = torch.cat(parts + digits[::-1], -1).to(self.dtype)
        gb = self.gate_mlp(ctrl)
        g, b = gb.split(self.n_kernels, -1)
        return torch.sigmoid(g), torch.tanh(b)

    def rbf_features(self, x: torch.Tensor) -> torch.Tensor:
        """Normalised per-cell RBF features ``[..., n_kernels]`` (before ``out_layer``)."""
        work = torch.float32 if x.device.type == "mps" else torch.float64
        xw = x.to(work)
        if self.gate_mlp is not None:
            m, e = scientific_decompose(xw, self.max_exp)
        else:
            m, e = xw, None
        diff = m.unsqueeze(-1) - self.centers.to(work)
        rbf = torch.exp(-(diff**2) / (2 * self.sigma.to(work) ** 2)).to(self.dtype)
        if self.gate_mlp is not None:
            g, b = self.control_table()
            idx = (xw < 0).long() * (2 * self.max_exp + 1) + (e + self.max_exp)
            # Select each cell's (gamma, beta) row with a one-hot product rather than a gather:
            # the values are identical (exact fp32 selection), but the backward pass becomes
            # one small GEMM instead of millions of contended index-accumulations into a
            # 38-row table.
            gb = torch.cat((g, b), -1)
            oh = torch.nn.functional.one_hot(idx, gb.shape[0]).to(gb.dtype)
            with torch.autocast(device_type=x.device.type, enabled=False):
                sel = oh @ gb
            gs, bs = sel.split(self.n_kernels, -1)
            rbf = rbf * gs + bs
            rbf = self.norm(rbf)
        if self.use_original_features:
            rbf = torch.cat([rbf, x.unsqueeze(-1).to(rbf.dtype)], -1)
        return rbf

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x.squeeze(-1)
        out = self.out_layer(self.rbf_features(x).to(self.dtype))
        return out if self.as_tokenizer else out.reshape(x.shape[0], -1)


class PBLDEmbedding(nn.Module):
    """Periodic + linear + dense cell embedding (reference ``model/encoders.py:279-306``)."""

    def __init__(self, embedding_size=96, n_frequencies=48, as_tokenizer=False, dtype=torch.float32):
        super().__init__()
        self.as_tokenizer = as_tokenizer
        self.n_frequencies = n_frequencies
        self.freq_weight = nn.Parameter(torch.randn(n_frequencies) * 0.5)
        self.freq_bias = nn.Parameter(torch.zeros(n_frequencies))
        self.periodic_dense = nn.Linear(n_frequencies, n_frequencies, dtype=dtype)
        self.periodic_norm = nn.LayerNorm(n_frequencies, dtype=dtype)
        self.out_layer = nn.Linear(n_frequencies + 1, embedding_size, dtype=dtype)

    def forward(self, x):
        x = x.squeeze(-1)
        p = torch.cos(2 * math.pi * self.freq_weight * x.unsqueeze(-1) + self.freq_bias)
        p = self.periodic_norm(self.periodic_dense(p) + p)
        out = self.out_layer(torch.cat([x.unsqueeze(-1), p], -1))
        return out if self.as_tokenizer else out.reshape(x.shape[0], -1)


class MaskEmbEncoder(nn.Module):
    """Per-cell numeric embedding (missing cells -> one learned vector), then the
    per-group fusion MLP ``fpg*E -> E -> E`` with LayerNorms."""

    def __init__(
        self,
        num_features: int,
        emsize: int,
        mask_embedding_size: int,
        numeric_embed_type: str = "linear",
        RBF_config: dict | None = None,
        PBLD_config: dict | None = None,
        prompt_quantile_ple_bins: int = 0,
        nan_to_zero: bool = False,
        bias: bool = True,
        in_keys=("data",),
        out_key: str = "data",
    ):
        super().__init__()
        self.embedding_dim = emsize
        self.mask_embedding_size = mask_embedding_size
        self.in_keys = list(in_keys)
        self.out_key = out_key
        self.prompt_quantile_ple_bins = int(prompt_quantile_ple_bins)
        if self.prompt_quantile_ple_bins in (1,) or self.prompt_quantile_ple_bins < 0:
            raise ValueError("prompt_quantile_ple_bins must be 0 or >= 2")
        if self.prompt_quantile_ple_bins >= emsize:
            raise ValueError("prompt_quantile_ple_bins must be smaller than the embedding dimension")
        num_dim = emsize - self.prompt_quantile_ple_bins
        self.mask_embedding = nn.Parameter(torch.randn(mask_embedding_size))
        self.numeric_embed_type = numeric_embed_type
        if numeric_embed_type == "linear":
            self.numeric_mlp = nn.Sequential(
                nn.Linear(1, emsize // 2, bias=bias),
                nn.LayerNorm(emsize // 2),
                nn.ReLU(),
                nn.Linear(emsize // 2, emsize, bias=bias),
                nn.LayerNorm(emsize),
                nn.ReLU(),
            )
        elif numeric_embed_type == "RBF":
            cfg = dict(RBF_config or {})
            bad = {
                k: cfg[k]
                for k, ok in (("input_transform", "scientific"), ("compute_dtype", "float64"), ("use_raw_input_residual", False))
                if k in cfg and cfg[k] != ok
            }
            if bad:
                raise ValueError(f"Unsupported RBF_config options: {bad}")
            self.numeric_mlp = RBFembedding(
                embedding_size=num_dim,
                exponent_digits=1,
                token_embed_dim=cfg["token_embed_dim"],
                n_kernels=cfg["n_kernels"],
                sigma=cfg["sigma"],
                use_learn_sigma=cfg.get("use_learn_sigma", False),
                use_learn_embeddings=cfg.get("use_learn_embeddings", False),
                center_range=(0.0, 10.0),
                use_original_features=cfg.get("use_original_features", False),
                as_tokenizer=True,
            )
        elif numeric_embed_type == "PBLD":
            nf = (PBLD_config or {}).get("n_frequencies", 48)
            self.numeric_mlp = PBLDEmbedding(embedding_size=emsize, n_frequencies=nf, as_tokenizer=True)
        else:
            raise ValueError(f"Invalid numeric_embed_type: {numeric_embed_type}")
        self.fusion_network = nn.Sequential(
            nn.Linear(num_features * emsize, emsize, bias=bias),
            nn.LayerNorm(emsize),
            nn.ReLU(),
            nn.Linear(emsize, emsize, bias=bias),
            nn.LayerNorm(emsize),
        )
        self.nan_to_zero = nan_to_zero

    def cell_embed(self, x: torch.Tensor, d: dict | None = None) -> torch.Tensor:
        """x: ``[B, S, G, fpg]`` (NaN = missing) -> per-cell ``[B, S, G, fpg, E]``."""
        xe = x.unsqueeze(-1)
        miss = torch.isnan(xe)
        xe = xe.masked_fill(miss, 0.0)
        emb = self.numeric_mlp(xe)
        if self.prompt_quantile_ple_bins:
            ref = (d or {}).get(PromptQuantilePLE.reference_key)
            if not isinstance(ref, dict):
                raise TypeError("prompt-quantile PLE reference is required")
            emb = torch.cat((emb, PromptQuantilePLE.encode(xe.squeeze(-1), ref).to(emb.dtype)), -1)
        if not self.nan_to_zero:
            emb = torch.where(miss, self.mask_embedding.to(emb.dtype).expand_as(emb), emb)
        return emb

    def forward(self, d: dict) -> dict:
        x = torch.cat([d[k] for k in self.in_keys], -1)
        B, S, G, _ = x.shape
        emb = self.cell_embed(x, d)
        d[self.out_key] = self.fusion_network(emb.flatten(3)).view(B, S, G, -1)
        return d


def build_x_encoder(
    *,
    num_features: int,
    embedding_size: int,
    mask_embedding_size: int,
    encoder_use_bias: bool,
    numeric_embed_type: str = "linear",
    RBF_config: dict | None = None,
    PBLD_config: dict | None = None,
    prompt_quantile_ple_bins: int = 0,
    in_keys=("data",),
    nan_to_zero: bool = False,
) -> nn.Sequential:
    return nn.Sequential(
        MaskEmbEncoder(
            num_features=num_features * len(in_keys),
            emsize=embedding_size,
            mask_embedding_size=mask_embedding_size,
            numeric_embed_type=numeric_embed_type,
            RBF_config=RBF_config,
            PBLD_config=PBLD_config,
            prompt_quantile_ple_bins=prompt_quantile_ple_bins,
            nan_to_zero=nan_to_zero,
            bias=encoder_use_bias,
            in_keys=in_keys,
        )
    )


# --------------------------------------------------------------------------------------
# y encoders
# --------------------------------------------------------------------------------------


class LinearEncoder(nn.Module):
    def __init__(self, num_features: int, emsize: int, nan_to_zero=False, bias=True, in_keys=("data",), out_key="data"):
        super().__init__()
        self.layer = nn.Linear(num_features, emsize, bias=bias)
        self.nan_to_zero, self.in_keys, self.out_key = nan_to_zero, list(in_keys), out_key

    def forward(self, d: dict) -> dict:
        x = torch.cat([d[k] for k in self.in_keys], -1)
        if self.nan_to_zero:
            x = torch.nan_to_num(x, nan=0.0, posinf=0.0, neginf=0.0)
        d[self.out_key] = self.layer(x)
        return d


class MulticlassTargetEncoder(nn.Module):
    """Rank-remap class labels present in the context to 0..K-1."""

    MAX_CLASSES = 10

    def forward(self, d: dict) -> dict:
        x = d["data"]
        ep = d["eval_pos"]
        ids = torch.arange(self.MAX_CLASSES, device=x.device, dtype=x.dtype)
        present = (x[:, :ep, :] == ids).any(1)
        cum = present.long().cumsum(1)
        ranks = torch.zeros_like(cum)
        ranks[:, 1:] = cum[:, :-1]
        idx = x[:, :, 0].long().clamp(0, self.MAX_CLASSES - 1)
        d["data"] = torch.gather(ranks, 1, idx).unsqueeze(-1).to(x.dtype)
        return d


class EmbYEncoderStep(nn.Module):
    """Orthogonal class embeddings for context labels and one mask row for queries."""

    def __init__(self, *, emsize: int, n_classes: int = 10):
        super().__init__()
        ortho = torch.empty(n_classes + 1, emsize)
        nn.init.orthogonal_(ortho)
        self.y_embedding = nn.Embedding(n_classes, emsize)
        self.y_embedding.weight.data = ortho[:n_classes].clone()
        self.y_mask = nn.Embedding(1, emsize)
        self.y_mask.weight.data = ortho[n_classes:].clone()

    def forward(self, d: dict) -> dict:
        y = d["data"].int()
        ep = d["eval_pos"]
        tr = self.y_embedding(y[:, :ep])
        te = self.y_mask(torch.zeros_like(y[:, ep:]))
        d["data"] = torch.cat([tr, te], 1)
        return d


def build_reg_y_encoder(*, num_inputs: int, embedding_size: int, nan_handling_y_encoder: bool, max_num_classes: int = 10):
    steps: list[nn.Module] = []
    keys = ["data"]
    if nan_handling_y_encoder:
        steps.append(NanEncoder())
        keys.append("nan_encoding")
    steps.append(LinearEncoder(num_inputs * len(keys), embedding_size, nan_to_zero=not nan_handling_y_encoder, in_keys=keys))
    return nn.Sequential(*steps)


def build_cls_y_encoder(*, num_inputs: int, embedding_size: int, nan_handling_y_encoder: bool, max_num_classes: int):
    steps: list[nn.Module] = []
    if nan_handling_y_encoder:
        steps.append(NanEncoder())
    if max_num_classes >= 2:
        steps.append(MulticlassTargetEncoder())
    steps.append(EmbYEncoderStep(emsize=embedding_size, n_classes=max_num_classes))
    return nn.Sequential(*steps)


def encoder_kwargs(cfg: dict[str, Any], keys) -> dict[str, Any]:
    return {k: cfg[k] for k in keys if k in cfg}
