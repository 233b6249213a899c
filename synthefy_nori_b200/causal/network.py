"""NoriCausal network: one table -> directed edge logits over its columns (+ target).

Parity target: reference ``causal/_network.py:58-278``: the Nori input embedding (per-cell
RBF tokens with two values per token, the regression y token, the column-gated
target-aware bias), ``n_blocks`` blocks that attend across rows then across columns,
order-free row pooling (mean and standard deviation, projected), ``n_pooled_blocks``
column-only blocks, and a low-rank bilinear edge head with source / destination biases:
``logits = A(S) B(S)^T / sqrt(r) + src(S) + dst(S)^T``.  Parameter names are the
checkpoints' (``enc.backbone.*``, ``hyp.*``, ``head.*``, ``null_token``).

Inputs longer than ``max_rows`` rows are evenly subsampled.  On CUDA the blocks run
under bf16 autocast (fused scaled-dot-product attention inside ``nn.MultiheadAttention``).
"""

from __future__ import annotations

import math

import torch
from torch import nn

from synthefy_nori_b200.models.encoders import build_reg_y_encoder, build_x_encoder, build_x_preprocess

EMBED_DIM = 128
FEATURES_PER_GROUP = 2
UNUSED_PREFIXES = ("enc.backbone.cls_y_encoder.", "enc.backbone.cls_target_aware_embedding.",
                   "enc.backbone.cls_y_decoder.", "enc.backbone.reg_y_decoder.", "enc.backbone.feature_decoder.")


class _Backbone(nn.Module):
    def __init__(self):
        super().__init__()
        self.embed_dim = EMBED_DIM
        self.x_preprocess = build_x_preprocess(num_features=2, nan_handling_enabled=True, normalize_on_train_only=True,
                                               normalize_x=True, remove_outliers=False,
                                               normalize_by_used_features=True)
        self.encoder_x = build_x_encoder(num_features=2, embedding_size=EMBED_DIM, mask_embedding_size=EMBED_DIM,
                                         encoder_use_bias=True, numeric_embed_type="RBF",
                                         RBF_config={"token_embed_dim": 16, "n_kernels": 64, "sigma": 0.5,
                                                     "use_learn_sigma": False, "use_learn_embeddings": False,
                                                     "use_random_kernels": False, "use_original_features": False})
        self.reg_y_encoder = build_reg_y_encoder(num_inputs=1, embedding_size=EMBED_DIM, nan_handling_y_encoder=True,
                                                 max_num_classes=10)
        self.reg_target_aware_embedding = nn.Linear(1, EMBED_DIM)
        self.column_y_aware_alpha = nn.Parameter(torch.tensor(-5.0))

    def forward(self, x: torch.Tensor, y: torch.Tensor, eval_pos: int) -> torch.Tensor:
        """x ``[1, S, F]`` (F even), y ``[1, eval_pos]`` -> tokens ``[1, S, F/2 + 1, E]``."""
        b, s, f = x.shape
        d = {"data": x.reshape(b, s, f // 2, 2), "mask": torch.isnan(x).to(torch.int32).reshape(b, s, f // 2, 2),
             "eval_pos": eval_pos}
        pre = self.x_preprocess(d)
        pre["data"] = torch.where(pre["mask"].bool(), float("nan"), pre["data"])
        ex = self.encoder_x(pre)["data"]
        yc = torch.cat([y, y.new_full((b, s - y.shape[1]), float("nan"))], 1) if y.shape[1] < s else y
        pos = torch.arange(s, device=y.device)
        ym = torch.where(pos[None] >= eval_pos, torch.full_like(yc, float("nan")), yc).unsqueeze(-1)
        ey = self.reg_y_encoder({"data": ym, "eval_pos": eval_pos})["data"]
        ey = ey.squeeze(2) if ey.dim() == 4 else ey
        ctx = self.reg_target_aware_embedding(yc[:, :eval_pos].unsqueeze(-1).to(ex.dtype)).to(ex.dtype)
        bias = torch.cat([ctx, ctx.new_zeros(b, s - eval_pos, EMBED_DIM)], 1).unsqueeze(2)
        gate = torch.sigmoid((ex * bias).sum(-1) / math.sqrt(EMBED_DIM)).unsqueeze(-1)
        a = torch.sigmoid(self.column_y_aware_alpha).to(ex.dtype)
        ex = ex + (1.0 - a) * bias + a * bias * gate
        return torch.cat((ex, ey.unsqueeze(2).to(ex.dtype)), 2)


class InputEncoder(nn.Module):
    """(X [N, C], y [N]) -> tokens [N, C+1, E]: every column duplicated into one two-value
    group (one token per column), a dummy query row appended and dropped."""

    def __init__(self):
        super().__init__()
        self.backbone = _Backbone()

    def forward(self, X: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        n = X.shape[0]
        xg = torch.cat([X, X[:1]], 0).repeat_interleave(FEATURES_PER_GROUP, dim=1)[None]
        yb = torch.cat([y, y.new_zeros(1)])[None]
        return self.backbone(xg, yb[:, :n], eval_pos=n)[0, :n]


class _Attn(nn.Module):
    def __init__(self, d, nhead, ff_mult=2):
        super().__init__()
        self.attn = nn.MultiheadAttention(d, nhead, batch_first=True)
        self.n1, self.n2 = nn.LayerNorm(d), nn.LayerNorm(d)
        self.ff = nn.Sequential(nn.Linear(d, ff_mult * d), nn.GELU(), nn.Linear(ff_mult * d, d))

    def forward(self, z):
        h = self.n1(z)
        z = z + self.attn(h, h, h, need_weights=False)[0]
        return z + self.ff(self.n2(z))


class STBlock(nn.Module):
    """Attention across rows, an MLP, then attention across columns; ``[N, T, d]``."""

    def __init__(self, d, nhead):
        super().__init__()
        self.row, self.feat = _Attn(d, nhead), _Attn(d, nhead)
        self.norm = nn.LayerNorm(d)
        self.mlp = nn.Sequential(nn.Linear(d, 2 * d), nn.GELU(), nn.Linear(2 * d, d))

    def forward(self, z):
        z = self.row(z.transpose(0, 1)).transpose(0, 1)
        z = z + self.mlp(self.norm(z))
        return self.feat(z)


class RowPool(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.proj = nn.Linear(2 * d, d)

    def forward(self, z):
        return self.proj(torch.cat([z.mean(0), z.std(0, unbiased=False)], -1))


class GraphEncoder(nn.Module):
    def __init__(self, embed_dim=EMBED_DIM, d=128, nhead=4, n_blocks=3, n_pooled_blocks=2, max_rows=256):
        super().__init__()
        self.max_rows = max_rows
        self.inp = nn.Linear(embed_dim, d)
        self.blocks = nn.ModuleList([STBlock(d, nhead) for _ in range(n_blocks)])
        self.pool = RowPool(d)
        self.pooled_blocks = nn.ModuleList([_Attn(d, nhead) for _ in range(n_pooled_blocks)])
        self.out_norm = nn.LayerNorm(d)
        self.feat_head = nn.Linear(d, 1)  # in the checkpoints; not read by the edge head
        self.bias_head = nn.Linear(d, 1)

    def forward(self, Z):
        if Z.shape[0] > self.max_rows:
            Z = Z[torch.linspace(0, Z.shape[0] - 1, self.max_rows, device=Z.device).long()]
        z = self.inp(Z)
        for blk in self.blocks:
            z = blk(z)
        S = self.pool(z)[None]
        for blk in self.pooled_blocks:
            S = blk(S)
        return self.out_norm(S)[0]


class DAGHead(nn.Module):
    def __init__(self, d=128, r=64):
        super().__init__()
        self.r = r
        self.A, self.B = nn.Linear(d, r, bias=False), nn.Linear(d, r, bias=False)
        self.src, self.dst = nn.Linear(d, 1), nn.Linear(d, 1)

    def forward(self, S):
        return self.A(S) @ self.B(S).t() / math.sqrt(self.r) + self.src(S) + self.dst(S).t()


class NoriCausalNetwork(nn.Module):
    def __init__(self, d=352, r=176, nhead=4, n_blocks=6, n_pooled_blocks=15, max_rows=2048):
        super().__init__()
        self.enc = InputEncoder()
        self.hyp = GraphEncoder(EMBED_DIM, d, nhead, n_blocks, n_pooled_blocks, max_rows)
        self.head = DAGHead(d, r)
        self.null_token = nn.Parameter(torch.zeros(EMBED_DIM))
        self.max_rows = max_rows

    def forward(self, X: torch.Tensor, y: torch.Tensor, null_target: bool = False) -> torch.Tensor:
        """(X [N, C], y [N]) -> logits [C+1, C+1], ``[i, j]`` scores node i -> node j."""
        if len(X) > self.max_rows:
            idx = torch.linspace(0, len(X) - 1, self.max_rows, device=X.device).long()
            X, y = X[idx], y[idx]
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=X.is_cuda):
            z = self.enc(X, y)
            if null_target:
                z = z.clone()
                z[:, -1, :] = self.null_token.to(z.dtype)
            return self.head(self.hyp(z)).float()

    @classmethod
    def from_checkpoint(cls, path, device="cpu"):
        ck = torch.load(path, map_location=device, weights_only=True)
        net = cls(d=ck["d"], r=ck["r"], nhead=ck.get("nhead", 4), n_blocks=ck["n_blocks"],
                  n_pooled_blocks=ck.get("n_pooled_blocks", 2), max_rows=ck.get("max_rows", 1024))
        state = {k: v for k, v in ck["state_dict"].items() if not k.startswith(UNUSED_PREFIXES)}
        missing, unexpected = net.load_state_dict(state, strict=False)
        if missing or unexpected:
            raise ValueError(f"checkpoint does not match the NoriCausal network: missing={missing[:5]} "
                             f"unexpected={unexpected[:5]}")
        meta = {k: ck.get(k) for k in ("step", "d", "r", "n_blocks", "n_pooled_blocks", "nhead", "max_rows")}
        return net.to(device).eval(), meta
