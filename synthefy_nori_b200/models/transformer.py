"""The Nori model: ``FeaturesTransformer`` and the reusable ``ContextCache``.

Parity target: reference ``src/synthefy_nori/model/transformer.py`` -
``FeaturesTransformer.__init__`` 69-369 (same sub-module names, so released
checkpoints load strictly), ``forward`` 371-523, feature grouping 564-605, feature
positional embeddings 629-651 / 1141-1167, target-aware embedding 1080-1132,
``build_context_cache`` 813-959, ``apply_context_cache`` 961-1078 (adaptive
query-chunk halving on OOM), ``forward_cached_regression`` 716-811.

Execution: on CUDA with the native extension loaded, the encoder stack runs the
fused B200 layer (``synthefy_nori_b200/ops/fused_layer.py``) and the cell embedding
runs the ``feature_embed`` kernel; the code below is the reference-semantics path
used on CPU and as the oracle in tests.  ``self.impl`` selects: ``"auto"`` (native
on CUDA), ``"native"`` (fail loudly without the extension) or ``"torch"``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Callable, Literal

import torch
import torch.nn as nn

from synthefy_nori_b200.models.encoders import (
    build_cls_y_encoder,
    build_reg_y_encoder,
    build_x_encoder,
    build_x_preprocess,
)
from synthefy_nori_b200.models.layers import EncoderBaseLayer, LayerStack, RMSNorm


@dataclass
class ContextCache:
    """Everything query rows need from a fixed context: per-layer cross K/V (bf16 dict
    or ``QuantizedKV``), frozen preprocessing statistics, the feature positional
    embedding drawn for this context, context targets and the row count."""

    caches: list
    feature_pos_emb: torch.Tensor | None
    norm_stats: dict | None
    y_train: torch.Tensor
    eval_pos: int
    nan_mean: torch.Tensor | None = None
    valid_feature_num: torch.Tensor | None = None
    query_y_embedding: torch.Tensor | None = None

    def nbytes(self) -> int:
        total = 0
        for c in self.caches:
            kv = c["seq_kv"]
            total += kv.nbytes() if hasattr(kv, "nbytes") else kv["kv"].numel() * kv["kv"].element_size()
        return total


def _native_cache_available() -> bool:
    from synthefy_nori_b200.ops import fused_layer

    return hasattr(fused_layer, "build_stack_cache")


class FeaturesTransformer(nn.Module):
    def __init__(
        self,
        *,
        preprocess_config_x: dict[str, Any],
        encoder_config_x: dict[str, Any],
        encoder_config_y: dict[str, Any],
        decoder_config: dict[str, Any],
        nlayers: int,
        nhead: int,
        embed_dim: int,
        hid_dim: int,
        feature_positional_embedding_type: str | None = "subortho",
        feature_positional_embedding_num_slots: int = 1000,
        mask_prediction: bool = False,
        features_per_group: int = 2,
        dropout: float = 0.0,
        pre_norm: bool = False,
        activation: str = "gelu",
        layer_norm_eps: float = 1e-5,
        device=None,
        dtype=None,
        recompute_attn: bool = False,
        mlp_use_residual: bool = False,
        layer_arch: str = "fmfmsm",
        norm_type: str = "layernorm",
        deepnorm_alpha: float | None = None,
        use_target_aware_embedding: bool = False,
        use_column_specific_y_aware: bool = False,
        use_logn_attention: bool = False,
        use_learnable_attn_temperature: bool = False,
        attn_n_ref: float = 1024.0,
        omit_feature_decoder: bool = False,
        two_phase_config: dict[str, Any] | None = None,
        **layer_kwargs: Any,
    ):
        super().__init__()
        if mlp_use_residual:
            raise ValueError("mlp_use_residual=True is unsupported")
        self.preprocess_config_x = preprocess_config_x
        self.encoder_config_x = encoder_config_x
        self.encoder_config_y = encoder_config_y
        self.decoder_config = decoder_config
        self.feature_positional_embedding_type = feature_positional_embedding_type
        self.nlayers, self.nhead, self.embed_dim, self.hid_dim = nlayers, nhead, embed_dim, hid_dim
        self.mask_prediction = mask_prediction
        self.features_per_group = int(features_per_group)
        if self.features_per_group < 1:
            raise ValueError("features_per_group must be at least 1")
        self.dropout, self.pre_norm, self.activation = dropout, pre_norm, activation
        self.layer_norm_eps, self.layer_arch, self.norm_type = layer_norm_eps, layer_arch, norm_type
        self.deepnorm_alpha = deepnorm_alpha
        self.omit_feature_decoder = bool(omit_feature_decoder)
        self.two_phase_config = dict(two_phase_config) if two_phase_config else None
        self.layer_kwargs = dict(layer_kwargs)
        self.impl = "auto"
        self._skip_feature_decoder = False

        # ---- regression head metadata (reference transformer.py:143-218)
        self.num_reg_quantiles = int(decoder_config.get("num_reg_quantiles", 1))
        loss = decoder_config.get("regression_loss")
        if loss is None:
            loss = "mse" if self.num_reg_quantiles == 1 else "pinball"
        self.regression_loss = str(loss)
        qs = decoder_config.get("regression_quantiles")
        if self.regression_loss == "pinball":
            if qs is None:
                self.regression_quantiles = tuple((i + 1.0) / (self.num_reg_quantiles + 1.0) for i in range(self.num_reg_quantiles))
            else:
                self.regression_quantiles = tuple(float(q) for q in qs)
                if len(self.regression_quantiles) != self.num_reg_quantiles:
                    raise ValueError("decoder_config.regression_quantiles length does not match num_reg_quantiles")
                rq = self.regression_quantiles
                if any(not math.isfinite(q) or q <= 0 or q >= 1 for q in rq) or any(a >= b for a, b in zip(rq, rq[1:])):
                    raise ValueError("decoder_config.regression_quantiles must be strictly increasing values in (0, 1)")
        else:
            self.regression_quantiles = ()
        self.num_bars = int(decoder_config.get("num_bars", self.num_reg_quantiles))
        self.bar_borders_low = float(decoder_config.get("bar_borders_low", -10.0))
        self.bar_borders_high = float(decoder_config.get("bar_borders_high", 10.0))
        self.bar_borders_mode = str(decoder_config.get("bar_borders_mode", "uniform"))
        if self.regression_loss == "bar_distribution":
            if self.bar_borders_mode == "normal_quantile":
                from scipy.stats import norm as _norm

                e = _norm.ppf(torch.linspace(0.0, 1.0, self.num_bars + 1).numpy())
                e[0], e[-1] = -8.0, 8.0
                borders = torch.from_numpy(e).float()
            else:
                borders = torch.linspace(self.bar_borders_low, self.bar_borders_high, self.num_bars + 1)
            self.register_buffer("bar_borders_buffer", borders, persistent=True)
        else:
            self.bar_borders_buffer = None

        # ---- target-aware embedding
        self.use_target_aware_embedding = use_target_aware_embedding
        self.use_column_specific_y_aware = use_column_specific_y_aware
        self.column_y_aware_alpha = (
            nn.Parameter(torch.tensor(-5.0, device=device, dtype=dtype or torch.float32)) if use_column_specific_y_aware else None
        )
        self.target_aware_scale = 1.0
        self.max_num_classes = int(encoder_config_y.get("max_num_classes", decoder_config.get("num_classes", 10)))
        self.use_logn_attention = use_logn_attention
        self.use_learnable_attn_temperature = use_learnable_attn_temperature
        self.attn_n_ref = float(attn_n_ref)

        def make_layer():
            return EncoderBaseLayer(
                embed_dim=embed_dim,
                hid_dim=hid_dim,
                nhead=nhead,
                dropout=dropout,
                pre_norm=pre_norm,
                activation=activation,
                layer_norm_eps=layer_norm_eps,
                device=device,
                dtype=dtype,
                recompute_attn=recompute_attn,
                layer_arch=layer_arch,
                norm_type=norm_type,
                deepnorm_alpha=deepnorm_alpha,
                use_logn_attention=use_logn_attention,
                use_learnable_attn_temperature=use_learnable_attn_temperature,
                attn_n_ref=attn_n_ref,
                **layer_kwargs,
            )

        self.encoder_x = build_x_encoder(**encoder_config_x)
        self.cls_y_encoder = build_cls_y_encoder(**encoder_config_y) if self.two_phase_config is None else None
        self.reg_y_encoder = build_reg_y_encoder(**encoder_config_y)
        if use_target_aware_embedding:
            self.cls_target_aware_embedding = (
                nn.Embedding(self.max_num_classes, embed_dim, device=device, dtype=dtype) if self.two_phase_config is None else None
            )
            self.reg_target_aware_embedding = nn.Linear(1, embed_dim, device=device, dtype=dtype)
            if self.cls_target_aware_embedding is not None:
                nn.init.normal_(self.cls_target_aware_embedding.weight, std=0.02)
            nn.init.normal_(self.reg_target_aware_embedding.weight, std=0.02)
            nn.init.zeros_(self.reg_target_aware_embedding.bias)
        else:
            self.cls_target_aware_embedding = None
            self.reg_target_aware_embedding = None

        if self.two_phase_config is None:
            self.transformer_encoder = LayerStack([make_layer() for _ in range(nlayers)])
            dec_in = embed_dim
        else:
            from synthefy_nori_b200.models.two_phase import TwoPhaseEncoder

            tp = self.two_phase_config
            self.transformer_encoder = TwoPhaseEncoder(
                embed_dim,
                nhead,
                hid_dim,
                target_tokens=int(tp["target_tokens"]),
                cell_layers=nlayers,
                row_layers=int(tp["row_layers"]),
                row_heads=int(tp["row_heads"]),
                row_hidden_dim=int(tp["row_hidden_dim"]),
                task_type="reg",
                max_num_classes=self.max_num_classes,
                layer_norm_eps=layer_norm_eps,
                device=device,
                dtype=dtype,
            )
            for p in self.reg_y_encoder.parameters():
                p.requires_grad_(False)
            dec_in = self.transformer_encoder.width
        self.supports_context_cache = self.two_phase_config is None
        if pre_norm:
            self.encoder_out_norm = (
                RMSNorm(embed_dim, eps=layer_norm_eps, elementwise_affine=False)
                if norm_type == "rmsnorm"
                else nn.LayerNorm(embed_dim, eps=layer_norm_eps, elementwise_affine=False)
            )
        else:
            self.encoder_out_norm = nn.Identity()
        self.cls_y_decoder = (
            nn.Sequential(nn.Linear(embed_dim, hid_dim), nn.GELU(), nn.Linear(hid_dim, decoder_config["num_classes"]))
            if self.two_phase_config is None
            else None
        )
        self.reg_y_decoder = nn.Sequential(
            nn.Linear(dec_in, hid_dim), nn.LayerNorm(hid_dim), nn.GELU(), nn.Linear(hid_dim, self.num_reg_quantiles)
        )
        self.feature_decoder = (
            None
            if self.omit_feature_decoder
            else nn.Sequential(nn.Linear(embed_dim, hid_dim), nn.LayerNorm(hid_dim), nn.GELU(), nn.Linear(hid_dim, self.features_per_group))
        )
        if feature_positional_embedding_type == "learned":
            self.feature_positional_embedding = nn.Embedding(feature_positional_embedding_num_slots, embed_dim)
            nn.init.normal_(self.feature_positional_embedding.weight, std=0.02)
            self.feature_positional_embedding_num_slots = feature_positional_embedding_num_slots
        elif feature_positional_embedding_type == "subortho":
            self.feature_positional_embedding = nn.Linear(embed_dim // 4, embed_dim)
        self.x_preprocess = build_x_preprocess(**preprocess_config_x)

    def load_state_dict(self, state_dict, strict: bool = True, assign: bool = False):
        """Load weights and invalidate the native path's cached bf16 weight layouts."""
        result = super().load_state_dict(state_dict, strict=strict, assign=assign)
        from synthefy_nori_b200.ops.fused_layer import bump_weight_generation

        bump_weight_generation()
        ref = getattr(self, "_nori_layout_owner", None)
        owner = ref() if ref is not None else None
        if owner is not None:  # a trainer's persistent bf16 layouts: refresh them from the new weights
            owner.resync_layouts()
        return result

    # ------------------------------------------------------------------ dispatch
    def use_native_two_phase(self, device: torch.device) -> bool:
        """The two-phase encoder runs on the native kernels for inference (no autograd) on
        CUDA when its dimensions fit them; training and other shapes use the module."""
        if self.two_phase_config is None or self.impl == "torch" or device.type != "cuda" or torch.is_grad_enabled():
            return False
        from synthefy_nori_b200 import ops

        if not ops.native_available():
            raise RuntimeError(
                "synthefy_nori_b200 native extension is not built; run `python setup.py build_ext --inplace` "
                f"(import error: {ops.native_import_error()})"
            )
        from synthefy_nori_b200.ops import two_phase as native_two_phase

        ok = native_two_phase.supported(self.transformer_encoder)
        if not ok and self.impl == "native":
            raise NotImplementedError("impl='native': the native kernels do not cover this two-phase encoder")
        return ok

    def use_native(self, device: torch.device) -> bool:
        if self.impl == "torch":
            return False
        if device.type != "cuda":
            if self.impl == "native":
                raise RuntimeError("impl='native' requires CUDA tensors")
            return False
        from synthefy_nori_b200 import ops

        if not ops.native_available():
            raise RuntimeError(
                "synthefy_nori_b200 native extension is not built; run `python setup.py build_ext --inplace` "
                f"(import error: {ops.native_import_error()})"
            )
        if self.two_phase_config is not None:
            return False
        from synthefy_nori_b200.ops.fused_layer import model_supported

        if not model_supported(self):
            if self.impl == "native":
                raise NotImplementedError("impl='native': the native kernels do not cover this layer variant")
            if not getattr(self, "_nori_warned_variant", False):
                import warnings

                warnings.warn("the native sm_100a kernels do not cover this encoder-layer variant (qk-norm in the "
                              "one-phase encoder, a LayerNorm layer, a head wider than 64, the fmfmsm arch or "
                              "post-norm); running the PyTorch path", RuntimeWarning, stacklevel=3)
                self._nori_warned_variant = True
            return False
        return True

    # ------------------------------------------------------------------ inputs
    def _build_x_preprocess_inputs(self, x: torch.Tensor, eval_pos: int):
        B, S, F = x.shape
        d: dict[str, Any] = {"data": x, "mask": (~torch.isfinite(x)).to(torch.int32)}
        pad = (-F) % self.features_per_group
        if pad:
            for k in ("data", "mask"):
                d[k] = torch.cat((d[k], d[k].new_zeros(B, S, pad)), -1)
        for k in ("data", "mask"):
            d[k] = d[k].reshape(B, S, -1, self.features_per_group)
        d["eval_pos"] = eval_pos
        return d, pad

    @staticmethod
    def process_4_x(d: dict) -> dict:
        d["data"] = torch.where(d["mask"].bool(), float("nan"), d["data"])
        return d

    def make_feature_positional_embeddings(self, n_groups, *, device, dtype):
        t = self.feature_positional_embedding_type
        if t == "subortho":
            with torch.autocast(device_type=device.type, enabled=False):
                e = torch.randn((n_groups, self.embed_dim // 4), device=device, dtype=torch.float32)
                nn.init.orthogonal_(e)
            return self.feature_positional_embedding(e.to(dtype))
        if t == "learned":
            idx = torch.randperm(self.feature_positional_embedding_num_slots, device=device)[:n_groups]
            return self.feature_positional_embedding(idx).to(dtype)
        if t is None or t == "none":
            return None
        raise ValueError(f"Unknown feature_positional_embedding_type={t}")

    def _encode_y(self, y: torch.Tensor, total_rows: int, eval_pos: int, task_type: str):
        """y ``[B, L]`` -> (raw targets padded with NaN to ``total_rows``, y token ``[B, total, E]``)."""
        y = y.unsqueeze(-1)
        if y.shape[1] < total_rows:
            y = torch.cat((y, torch.full((y.shape[0], total_rows - y.shape[1], 1), float("nan"), device=y.device, dtype=y.dtype)), 1)
        raw = y.squeeze(-1).clone()
        pos = torch.arange(total_rows, device=y.device).view(1, -1, 1)
        masked = torch.where(pos >= eval_pos, torch.full_like(y, float("nan")), y)
        enc = self.cls_y_encoder if task_type == "cls" else self.reg_y_encoder
        emb = enc({"data": masked, "eval_pos": eval_pos})["data"]
        if emb.dim() == 4:
            emb = emb.squeeze(2)
        return raw, emb, masked.squeeze(-1)

    def apply_target_aware_embedding(self, x, y, *, task_type, eval_pos):
        scale = float(getattr(self, "target_aware_scale", 1.0))
        if not self.use_target_aware_embedding or eval_pos <= 0 or abs(scale) < 1e-8:
            return x
        if task_type == "cls":
            yc = torch.clamp(y[:, :eval_pos].long(), 0, self.max_num_classes - 1)
            bias = self.cls_target_aware_embedding(yc).to(x.dtype)
        else:
            bias = self.reg_target_aware_embedding(y[:, :eval_pos].unsqueeze(-1).to(x.dtype)).to(x.dtype)
        bias = torch.cat([bias, bias.new_zeros(x.shape[0], x.shape[1] - eval_pos, self.embed_dim)], 1)
        if scale != 1.0:
            bias = bias * scale
        rb = bias.unsqueeze(2)
        if self.use_column_specific_y_aware and self.column_y_aware_alpha is not None:
            gate = torch.sigmoid((x * rb).sum(-1) / math.sqrt(self.embed_dim)).unsqueeze(-1)
            a = torch.sigmoid(self.column_y_aware_alpha).to(x.dtype)
            return x + (1.0 - a) * rb + a * (rb * gate)
        return x + rb

    def encode_cells(self, preprocessed: dict) -> torch.Tensor:
        """Per-group token embedding ``[B, S, G, E]`` of preprocessed x."""
        return self.encoder_x(preprocessed)["data"]

    def embed(self, x, y, eval_pos, task_type="reg", feature_pos_emb=None):
        """Token tensor ``[B, S, G+1, E]`` plus preprocessing side outputs."""
        S = x.shape[1]
        d, pad = self._build_x_preprocess_inputs(x, eval_pos)
        pre = self.process_4_x(self.x_preprocess(d))
        xe = self.encode_cells(pre)
        raw_y, ye, masked_y = self._encode_y(y, S, eval_pos, task_type)
        if feature_pos_emb is None and self.feature_positional_embedding_type not in (None, "none"):
            feature_pos_emb = self.make_feature_positional_embeddings(xe.shape[2], device=xe.device, dtype=xe.dtype)
        if feature_pos_emb is not None:
            xe = xe + feature_pos_emb[None, None]
        xe = self.apply_target_aware_embedding(xe, raw_y, task_type=task_type, eval_pos=eval_pos)
        return xe, ye, pre, pad, masked_y

    # ------------------------------------------------------------------ forward
    def run_encoder(self, tokens: torch.Tensor, eval_pos: int) -> torch.Tensor:
        if self.use_native(tokens.device):
            from synthefy_nori_b200.ops.fused_layer import run_stack

            return run_stack(self, tokens, eval_pos)
        return self.transformer_encoder(tokens, feature_atten_mask=None, eval_pos=eval_pos)[0]

    def forward(
        self,
        x: torch.Tensor,
        y: torch.Tensor,
        eval_pos: int,
        y_type=None,
        task_type: Literal["reg", "cls"] = "cls",
        return_embeddings: bool = False,
        **kwargs,
    ):
        assert x is not None and y is not None, "x and y must not be none"
        assert eval_pos > 0, "eval_pos must be a positive number"
        assert x.dim() == 3 and y.dim() == 2
        assert eval_pos < x.shape[1] and eval_pos <= y.shape[1], "invalid eval_pos"
        if self.two_phase_config is not None and task_type != "reg":
            raise ValueError("the two-phase encoder supports regression only; pass task_type='reg'")
        xe, ye, pre, pad, masked_y = self.embed(x, y, eval_pos, task_type)
        if self.two_phase_config is not None:
            if self.use_native_two_phase(xe.device):
                from synthefy_nori_b200.ops import two_phase as native_two_phase

                rows, cells = native_two_phase.forward(self.transformer_encoder, xe, masked_y, eval_pos)
                rows, cells = rows.to(xe.dtype), cells.to(xe.dtype)
            else:
                rows, cells = self.transformer_encoder(xe, masked_y, eval_pos)
            if return_embeddings:
                return rows
            reg = self.reg_y_decoder(rows[:, eval_pos:])
            if not self.mask_prediction:
                return reg
            fp = None if (self.feature_decoder is None or self._skip_feature_decoder) else self.feature_decoder(cells)
            return {"reg_output": reg, "feature_pred": fp, "process_config": self._process_config(pre, pad)}
        tokens = torch.cat((xe, ye.unsqueeze(2).to(xe.dtype)), 2)
        out = self.encoder_out_norm(self.run_encoder(tokens, eval_pos))
        if return_embeddings:
            return out[:, :, -1]
        target = out[:, eval_pos:, -1]
        if self.mask_prediction:
            if task_type == "cls":
                cls_out = self.cls_y_decoder(target)
                reg_out = target.new_zeros(*target.shape[:2], self.num_reg_quantiles)
            else:
                cls_out = target.new_zeros(*target.shape[:2], self.cls_y_decoder[-1].out_features)
                reg_out = self.decode_regression(target)
            fp = None if (self.feature_decoder is None or self._skip_feature_decoder) else self.feature_decoder(out[:, :, :-1])
            return {"cls_output": cls_out, "reg_output": reg_out, "feature_pred": fp, "process_config": self._process_config(pre, pad)}
        return self.cls_y_decoder(target) if task_type == "cls" else self.decode_regression(target)

    def decode_regression(self, h: torch.Tensor) -> torch.Tensor:
        return self.reg_y_decoder(h)

    def _process_config(self, pre, pad):
        return {
            "n_x_padding": pad,
            "features_per_group": self.features_per_group,
            "num_used_features": pre.get("_valid_feature_num"),
            "mean_for_normalization": pre.get("_norm_mean"),
            "std_for_normalization": pre.get("_norm_std"),
        }

    # ------------------------------------------------------------------ context cache
    def build_context_cache(self, x_train, y_train, *, cache_dtype: str = "bf16", fit_row_chunk=None,
                            placement: str = "resident", stream_block_rows: int | None = None, **_) -> ContextCache:
        """Per-layer cross-attention K/V of the context rows.  ``placement``: ``"resident"``
        (device), ``"offload"`` (pinned host, one layer copied in at a time) or
        ``"stream"`` (pinned host in blocks of ``stream_block_rows`` context rows, the
        query attention merging block partials) - the native path only."""
        if not self.supports_context_cache:
            raise NotImplementedError("context caching is not implemented for the two-phase encoder")
        if cache_dtype not in ("bf16", "int8"):
            raise ValueError(f"build_context_cache takes cache_dtype 'bf16' or 'int8', got {cache_dtype!r}")
        if self.mask_prediction:
            raise NotImplementedError("build_context_cache requires mask_prediction=False")
        tokens, context = self.context_tokens(x_train, y_train)
        if self.use_native(tokens.device) and _native_cache_available():
            from synthefy_nori_b200.ops.fused_layer import build_stack_cache

            caches = build_stack_cache(self, tokens, quantize=cache_dtype == "int8")
            if placement != "resident":
                from synthefy_nori_b200.ops.fused_layer import place_caches

                caches = place_caches(caches, placement, stream_block_rows)
        else:
            if placement != "resident":
                raise NotImplementedError("host-offloaded / streamed caches need the native CUDA path")
            _, caches = self.transformer_encoder.build_train_cache(tokens, quantize=cache_dtype == "int8")
        context.caches = caches
        return context

    def context_tokens(self, x_train, y_train) -> tuple[torch.Tensor, ContextCache]:
        """Embed the context rows: tokens ``[B, N, G+1, E]`` and a ``ContextCache`` holding
        everything query rows need except the per-layer K/V (``caches`` left empty)."""
        ep = x_train.shape[1]
        if ep <= 0 or y_train.shape[1] < ep:
            raise AssertionError("x_train must have context rows and y_train must cover them")
        d, _ = self._build_x_preprocess_inputs(x_train, ep)
        pre = self.x_preprocess(d)
        cap = pre.get("_norm_stats") or {}
        norm_stats = {k: v.detach() for k, v in cap.items()} or None
        nan_mean = pre.get("_nan_mean")
        vfn = pre.get("_valid_feature_num")
        pre = self.process_4_x(pre)
        xe = self.encode_cells(pre)
        fpe = self.make_feature_positional_embeddings(xe.shape[2], device=xe.device, dtype=xe.dtype)
        if fpe is not None:
            xe = xe + fpe[None, None]
        raw_y, ye, _ = self._encode_y(y_train[:, :ep], ep, ep, "reg")
        xe = self.apply_target_aware_embedding(xe, raw_y, task_type="reg", eval_pos=ep)
        tokens = torch.cat((xe, ye.unsqueeze(2).to(xe.dtype)), 2)
        ctx = ContextCache(
            caches=[],
            feature_pos_emb=fpe,
            norm_stats=norm_stats,
            y_train=y_train[:, :ep].detach(),
            eval_pos=ep,
            nan_mean=nan_mean.detach() if isinstance(nan_mean, torch.Tensor) else None,
            valid_feature_num=vfn.detach() if isinstance(vfn, torch.Tensor) else None,
        )
        return tokens, ctx

    def query_tokens(self, x_test, context: ContextCache) -> torch.Tensor:
        """Tokens ``[B, Nq, G+1, E]`` of query rows, preprocessed with the context's frozen
        statistics (the same construction ``apply_context_cache`` uses per chunk)."""
        ep, nq = context.eval_pos, x_test.shape[1]
        d, _ = self._build_x_preprocess_inputs(x_test, nq)
        if context.norm_stats is not None:
            d["_frozen_norm_stats"] = {k: v.to(x_test.device) for k, v in context.norm_stats.items()}
        if context.nan_mean is not None:
            d["_frozen_nan_mean"] = context.nan_mean.to(x_test.device)
        if context.valid_feature_num is not None:
            d["_frozen_valid_feature_num"] = context.valid_feature_num.to(x_test.device)
        pre = self.process_4_x(self.x_preprocess(d))
        xq = self.encode_cells(pre)
        if context.feature_pos_emb is not None:
            xq = xq + context.feature_pos_emb[None, None]
        if context.query_y_embedding is None:
            _, yfull, _ = self._encode_y(context.y_train, ep + nq, ep, "reg")
            yq = yfull[:, ep:]
        else:
            yq = context.query_y_embedding.expand(-1, nq, -1)
        return torch.cat((xq, yq.unsqueeze(2).to(xq.dtype)), 2)

    def apply_context_cache(
        self,
        x_test,
        context: ContextCache,
        *,
        row_chunk_size: int | None = None,
        adaptive_query_chunk: bool = True,
        query_chunk_attempt_callback: Callable[[int, str], None] | None = None,
        return_hidden: bool = False,
    ):
        if self.mask_prediction:
            raise NotImplementedError("apply_context_cache requires mask_prediction=False")
        ep, nq = context.eval_pos, x_test.shape[1]
        if nq <= 0:
            raise AssertionError("x_test must have at least one query row")
        d, _ = self._build_x_preprocess_inputs(x_test, nq)
        if context.norm_stats is not None:
            d["_frozen_norm_stats"] = {k: v.to(x_test.device) for k, v in context.norm_stats.items()}
        if context.nan_mean is not None:
            d["_frozen_nan_mean"] = context.nan_mean.to(x_test.device)
        if context.valid_feature_num is not None:
            d["_frozen_valid_feature_num"] = context.valid_feature_num.to(x_test.device)
        pre = self.process_4_x(self.x_preprocess(d))
        if context.query_y_embedding is None:
            _, yfull, _ = self._encode_y(context.y_train, ep + nq, ep, "reg")
            yq_all = yfull[:, ep:]
        native = self.use_native(x_test.device) and _native_cache_available()

        def run(s, e):
            part = {k: (v[:, s:e] if k in ("data", "mask") else v) for k, v in pre.items()}
            xq = self.encode_cells(part)
            if context.feature_pos_emb is not None:
                xq = xq + context.feature_pos_emb[None, None]
            yq = yq_all[:, s:e] if context.query_y_embedding is None else context.query_y_embedding.expand(-1, e - s, -1)
            tok = torch.cat((xq, yq.unsqueeze(2).to(xq.dtype)), 2)
            if native:
                from synthefy_nori_b200.ops.fused_layer import run_stack_cached

                h = run_stack_cached(self, tok, context.caches)
            else:
                h = self.transformer_encoder.forward_test_with_cache(tok, context.caches)
            h = self.encoder_out_norm(h)[:, :, -1]
            return h if return_hidden else self.decode_regression(h)

        chunk = nq if (row_chunk_size is None or row_chunk_size <= 0) else row_chunk_size
        outs, s = [], 0
        while s < nq:
            e = min(s + chunk, nq)
            try:
                outs.append(run(s, e))
                s = e
            except torch.cuda.OutOfMemoryError:
                if query_chunk_attempt_callback is not None:
                    query_chunk_attempt_callback(chunk, "oom")
                if not adaptive_query_chunk or chunk <= 1:
                    raise
                torch.cuda.empty_cache()
                chunk = max(1, chunk // 2)
        if query_chunk_attempt_callback is not None:
            query_chunk_attempt_callback(chunk, "success")
        return torch.cat(outs, 1)

    def forward_cached_regression(self, x, y, eval_pos, *, row_chunk_size=None, cache_dtype="bf16", adaptive_query_chunk=True, **kw):
        if self.two_phase_config is not None:
            raise NotImplementedError("context caching is not implemented for the two-phase encoder")
        if kw.get("quantize_kv_cache") is not None and cache_dtype == "bf16":
            cache_dtype = "int8" if kw["quantize_kv_cache"] else "bf16"
        bundle = self.build_context_cache(x[:, :eval_pos], y[:, :eval_pos], cache_dtype=cache_dtype)
        return self.apply_context_cache(x[:, eval_pos:], bundle, row_chunk_size=row_chunk_size, adaptive_query_chunk=adaptive_query_chunk)
