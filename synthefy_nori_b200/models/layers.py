"""Transformer building blocks of the Nori encoder (plain PyTorch path).

Parity targets (reference ``src/synthefy_nori/model/layer.py``):

* ``RMSNorm`` 233-258, ``LayerNormMixedPrecision`` 219-230;
* ``SwiGLUMLP`` 261-274 (hidden = int(2*H/3), no bias), ``MLP`` 277-313;
* ``QASSMaxScaling`` 316-456 (q * log n * (1+tanh(base(log n))) * (1+tanh(gate(q))));
* ``MultiheadAttention`` 459-1162 (weights ``qkv_proj_weight [3,H,D,E]``,
  ``out_proj_weight [H,D,E]``; log-n / learnable temperature pre-scaling of Q; MQA
  when ``copy_first_head_kv``; cached cross-attention over projected K/V);
* ``EncoderBaseLayer`` 1165-2027 (layer arches ``smf`` and ``fmfmsm``, pre-norm with a
  DeepNorm residual factor or post-norm, isolated self/cross sequence attention);
* ``LayerStack`` 2030-2108.

This file is the numerical oracle for the fused B200 layer in
``synthefy_nori_b200/ops/fused_layer.py``; the module and parameter names are the
reference checkpoint's state-dict keys.
"""

from __future__ import annotations

import math
from functools import partial
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint


ACTIVATIONS = {"gelu": nn.GELU, "relu": nn.ReLU, "silu": nn.SiLU}


class LayerNormMixedPrecision(nn.LayerNorm):
    """LayerNorm that runs outside fp16 autocast for widths below 512."""

    def forward(self, x):
        if x.dtype == torch.float16 and sum(self.normalized_shape) < 512:
            with torch.autocast(device_type=x.device.type, enabled=False):
                return super().forward(x)
        return super().forward(x)


class RMSNorm(nn.Module):
    def __init__(self, normalized_shape, eps=1e-5, elementwise_affine=False, device=None, dtype=None):
        super().__init__()
        if isinstance(normalized_shape, int):
            normalized_shape = (normalized_shape,)
        self.normalized_shape = tuple(normalized_shape)
        self.eps = eps
        self.elementwise_affine = elementwise_affine
        self.use_native = False
        if elementwise_affine:
            self.weight = nn.Parameter(torch.ones(self.normalized_shape, device=device, dtype=dtype))
        else:
            self.register_parameter("weight", None)

    def forward(self, x):
        if self.use_native:
            return F.rms_norm(x, self.normalized_shape, weight=self.weight, eps=self.eps)
        y = x * x.pow(2).mean(-1, keepdim=True).add(self.eps).rsqrt()
        return y * self.weight if self.weight is not None else y


class SwiGLUMLP(nn.Module):
    def __init__(self, in_features, hidden_size, out_features, has_bias, device, dtype):
        super().__init__()
        h = int(2 * hidden_size / 3)
        self.w_gate = nn.Linear(in_features, h, bias=has_bias, device=device, dtype=dtype)
        self.w_up = nn.Linear(in_features, h, bias=has_bias, device=device, dtype=dtype)
        self.w_down = nn.Linear(h, out_features, bias=has_bias, device=device, dtype=dtype)
        nn.init.normal_(self.w_down.weight, std=0.02)

    def forward(self, x):
        return self.w_down(F.silu(self.w_gate(x)) * self.w_up(x))


class MLP(nn.Module):
    def __init__(self, in_features, hidden_size, out_features, has_bias, device, dtype, activation="gelu", depth=2):
        super().__init__()
        self.in_features, self.out_features, self.activation = in_features, out_features, activation
        layers: list[nn.Module] = []
        if depth == 1:
            layers.append(nn.Linear(in_features, out_features, bias=has_bias, device=device, dtype=dtype))
        else:
            layers += [nn.Linear(in_features, hidden_size, bias=has_bias, device=device, dtype=dtype), ACTIVATIONS[activation]()]
            for _ in range(depth - 2):
                layers += [nn.Linear(hidden_size, hidden_size, bias=has_bias, device=device, dtype=dtype), ACTIVATIONS[activation]()]
            layers.append(nn.Linear(hidden_size, out_features, bias=has_bias, device=device, dtype=dtype))
            nn.init.normal_(layers[-1].weight, std=0.02)
        self.mlp = nn.Sequential(*layers)

    def forward(self, x):
        return self.mlp(x)


class QASSMaxScaling(nn.Module):
    """Query-aware scalable softmax as a rescaling of Q (modes full / base_only / log_only)."""

    def __init__(self, *, num_heads, head_dim, hidden_dim=64, qass_mode=None, device=None, dtype=None):
        super().__init__()
        import os

        self.num_heads, self.head_dim = num_heads, head_dim
        mode = qass_mode if qass_mode is not None else os.environ.get("SYNTHEFY_QASS_MODE", "full")
        self.qass_mode = str(mode).strip().lower()
        if self.qass_mode not in ("full", "base_only", "log_only"):
            raise ValueError(f"qass_mode must be full, base_only or log_only; got {self.qass_mode!r}")
        # Both MLPs are constructed in every mode so the RNG stream of a seeded init
        # matches the reference; unused ones are dropped.
        base = nn.Sequential(
            nn.Linear(1, hidden_dim, device=device, dtype=dtype), nn.GELU(), nn.Linear(hidden_dim, num_heads * head_dim, device=device, dtype=dtype)
        )
        gate = nn.Sequential(
            nn.Linear(head_dim, hidden_dim, device=device, dtype=dtype), nn.GELU(), nn.Linear(hidden_dim, head_dim, device=device, dtype=dtype)
        )
        self.base_mlp = base if self.qass_mode != "log_only" else None
        self.gate_mlp = gate if self.qass_mode == "full" else None
        for m in (self.base_mlp, self.gate_mlp):
            if m is not None:
                nn.init.zeros_(m[-1].weight)
                nn.init.zeros_(m[-1].bias)

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        drop = []
        if self.base_mlp is None:
            drop.append(prefix + "base_mlp.")
        if self.gate_mlp is None:
            drop.append(prefix + "gate_mlp.")
        if drop:
            state_dict = {k: v for k, v in state_dict.items() if not k.startswith(tuple(drop))}
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)

    def base_scale(self, key_len: int, dtype, device) -> torch.Tensor:
        """``[H, D]`` per-(head, dim) factor ``log n * (1 + tanh(base(log n)))``."""
        log_n = torch.tensor(math.log(float(max(key_len, 2))), device=device, dtype=dtype)
        if self.qass_mode == "log_only":
            return log_n.expand(self.num_heads, self.head_dim)
        delta = self.base_mlp(log_n.view(1, 1)).view(self.num_heads, self.head_dim)
        return log_n * (1.0 + torch.tanh(delta))

    def forward(self, q: torch.Tensor, key_len: int) -> torch.Tensor:
        if key_len <= 1:
            return q
        s = self.base_scale(key_len, q.dtype, q.device)
        out = q * s
        if self.qass_mode == "full":
            out = out * (1.0 + torch.tanh(self.gate_mlp(q)))
        return out


def sdpa(q, k, v, attn_mask=None, dropout_p=0.0):
    """q ``[B, Lq, H, D]``, k/v ``[B, Lk, Hkv, D]`` -> ``[B, Lq, H, D]``; Hkv == 1 broadcasts."""
    if k.shape[2] != q.shape[2]:
        k = k.expand(-1, -1, q.shape[2], -1)
        v = v.expand(-1, -1, q.shape[2], -1)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), attn_mask=attn_mask, dropout_p=dropout_p)
    return o.transpose(1, 2)


class MultiheadAttention(nn.Module):
    def __init__(
        self,
        embed_dim,
        num_heads,
        device=None,
        dtype=None,
        qkv_combined=True,
        dropout=0.0,
        recompute=False,
        use_qassmax=False,
        use_logn_attention=False,
        use_learnable_attn_temperature=False,
        attn_n_ref=1024.0,
        qass_mode=None,
        qk_norm=False,
        **_unused,
    ):
        super().__init__()
        assert embed_dim % num_heads == 0
        self.embed_dim, self.num_heads = embed_dim, num_heads
        self.head_dim = embed_dim // num_heads
        self.qkv_combined, self.dropout, self.recompute = qkv_combined, dropout, recompute
        self.use_qassmax = use_qassmax
        self.qk_norm = bool(qk_norm)
        if self.qk_norm:
            self.q_norm = RMSNorm(self.head_dim, eps=1e-6, elementwise_affine=True, device=device, dtype=dtype)
            self.k_norm = RMSNorm(self.head_dim, eps=1e-6, elementwise_affine=True, device=device, dtype=dtype)
        else:
            self.q_norm = self.k_norm = None
        self.use_logn_attention = use_logn_attention
        self.use_learnable_attn_temperature = use_learnable_attn_temperature
        self.attn_n_ref = float(attn_n_ref)
        self._log_n_ref = math.log(max(self.attn_n_ref, 2.0))
        self.attn_temperature = (
            nn.Parameter(torch.ones(1, device=device, dtype=dtype or torch.float32)) if use_learnable_attn_temperature else None
        )
        self.out_proj_weight = nn.Parameter(torch.empty(num_heads, self.head_dim, embed_dim, device=device, dtype=dtype))
        self.qkv_proj_weight = nn.Parameter(torch.empty(3, num_heads, self.head_dim, embed_dim, device=device, dtype=dtype))
        nn.init.normal_(self.out_proj_weight, std=0.02)
        nn.init.xavier_uniform_(self.qkv_proj_weight)
        self.qassmax = (
            QASSMaxScaling(num_heads=num_heads, head_dim=self.head_dim, hidden_dim=64, qass_mode=qass_mode, device=device, dtype=dtype)
            if use_qassmax
            else None
        )

    # ---------------------------------------------------------------- helpers
    def extra_q_scale(self, n_keys: int):
        """Multiplier folded into Q for log-n attention and the learnable temperature."""
        if not self.use_logn_attention and not self.use_learnable_attn_temperature:
            return None
        f: float | torch.Tensor = 1.0
        if self.use_logn_attention:
            f = math.log(max(int(n_keys), 2)) / self._log_n_ref
        if self.attn_temperature is not None:
            f = self.attn_temperature.abs() * f
        return f

    def scale_q(self, q, n_keys):
        if self.qassmax is not None:
            q = self.qassmax(q, n_keys)
        f = self.extra_q_scale(n_keys)
        return q if f is None else q * f

    def _drop_p(self):
        return float(self.dropout) if self.training else 0.0

    def project_q(self, x):
        q = torch.einsum("...e,hde->...hd", x, self.qkv_proj_weight[0])
        return self.q_norm(q) if self.q_norm is not None else q

    def project_kv(self, x, copy_first_head=False):
        w = self.qkv_proj_weight[1:]
        if copy_first_head:
            w = w[:, :1]
        kv = torch.einsum("...e,jhde->...jhd", x, w)
        if self.k_norm is not None:
            kv = torch.stack((self.k_norm(kv[..., 0, :, :]), kv[..., 1, :, :]), dim=-3)
        return kv

    def out_proj(self, o):
        return torch.einsum("...hd,hde->...e", o, self.out_proj_weight)

    # ---------------------------------------------------------------- forward
    def forward(self, x, x_kv=None, copy_first_head_kv=False, attn_mask=None, **_):
        """x ``[B, S, L, E]`` (attention over L); x_kv same layout for separate Q/KV."""
        B, S = x.shape[:2]
        xf = x.reshape(-1, *x.shape[-2:])
        if self.qkv_combined:
            qkv = torch.einsum("...e,jhde->...jhd", xf, self.qkv_proj_weight)
            q, k, v = qkv.unbind(-3)
            if self.qk_norm:
                q, k = self.q_norm(q), self.k_norm(k)
        else:
            kvf = x_kv.reshape(-1, *x_kv.shape[-2:])
            q = self.project_q(xf)
            k, v = self.project_kv(kvf, copy_first_head_kv).unbind(-3)
        q = self.scale_q(q, k.shape[1])
        o = sdpa(q, k, v, attn_mask=attn_mask, dropout_p=self._drop_p())
        out = self.out_proj(o)
        return out.reshape(B, S, *out.shape[1:]), None, None

    def project_kv_cache(self, x_kv, *, copy_first_head_kv=False):
        """Project context K/V once: x_kv ``[B, G, N, E]`` -> ``{"kv": [B*G, N, 2, Hkv, D]}``."""
        B, G = x_kv.shape[:2]
        kv = self.project_kv(x_kv.reshape(-1, *x_kv.shape[-2:]), copy_first_head_kv)
        return {"kv": kv.contiguous(), "batch": B, "groups": G}

    def forward_with_kv_cache(self, x, kv_cache):
        """Cross-attention of query rows x ``[B, G, Nq, E]`` against a projected cache."""
        from synthefy_nori_b200.models.kv_cache import QuantizedKV

        B, G = x.shape[:2]
        xf = x.reshape(-1, *x.shape[-2:])
        q = self.project_q(xf)
        if isinstance(kv_cache, QuantizedKV):
            n_keys = kv_cache.n_rows
            q = self.scale_q(q, n_keys)
            o = kv_cache.attend(q)
        else:
            kv = kv_cache["kv"]
            n_keys = kv.shape[1]
            q = self.scale_q(q, n_keys)
            k, v = kv.unbind(2)
            o = sdpa(q, k, v)
        out = self.out_proj(o)
        return out.reshape(B, G, *out.shape[1:]), None


class EncoderBaseLayer(nn.Module):
    def __init__(
        self,
        nhead,
        embed_dim,
        hid_dim,
        dropout=0.0,
        pre_norm=False,
        activation="gelu",
        layer_norm_eps=1e-5,
        device=None,
        dtype=None,
        recompute_attn=False,
        mlp_use_residual=False,
        layer_arch="fmfmsm",
        seq_attn_isolated=False,
        seq_attn_serial=False,
        self_share_all_kv_heads=False,
        cross_share_all_kv_heads=True,
        use_qassmax=False,
        norm_type="layernorm",
        deepnorm_alpha=None,
        use_logn_attention=False,
        use_learnable_attn_temperature=False,
        attn_n_ref=1024.0,
        qass_mode=None,
    ):
        super().__init__()
        if mlp_use_residual:
            raise ValueError("mlp_use_residual=True is unsupported (the outer residual already applies)")
        self.nhead, self.embed_dim, self.hid_dim = nhead, embed_dim, hid_dim
        self.pre_norm, self.activation, self.layer_norm_eps = pre_norm, activation, layer_norm_eps
        self.layer_arch, self.norm_type = layer_arch, norm_type
        self.head_dim = embed_dim // nhead
        self.self_share_all_kv_heads = self_share_all_kv_heads
        self.cross_share_all_kv_heads = cross_share_all_kv_heads
        self.seq_attn_serial, self.seq_attn_isolated = seq_attn_serial, seq_attn_isolated
        self.use_qassmax = use_qassmax
        n_feat, n_mlp = (2, 3) if layer_arch == "fmfmsm" else (1, 1)
        if layer_arch not in ("fmfmsm", "smf"):
            raise ValueError(f"Unsupported layer arch: {layer_arch}")
        n_seq = 2 if seq_attn_isolated else 1
        if deepnorm_alpha is not None:
            self.register_buffer("deepnorm_alpha", torch.tensor(deepnorm_alpha, dtype=torch.float32))
        else:
            self.deepnorm_alpha = None
        common = dict(
            embed_dim=embed_dim,
            num_heads=nhead,
            device=device,
            dtype=dtype,
            dropout=dropout,
            recompute=recompute_attn,
            use_logn_attention=use_logn_attention,
            use_learnable_attn_temperature=use_learnable_attn_temperature,
            attn_n_ref=attn_n_ref,
        )
        self.feature_attentions = nn.ModuleList([MultiheadAttention(qkv_combined=True, use_qassmax=False, **common) for _ in range(n_feat)])
        self.sequence_attentions = nn.ModuleList(
            [MultiheadAttention(qkv_combined=False, use_qassmax=use_qassmax, qass_mode=qass_mode, **common) for _ in range(n_seq)]
        )
        if activation == "swiglu":
            mk = lambda: SwiGLUMLP(embed_dim, hid_dim, embed_dim, False, device, dtype)  # noqa: E731
        else:
            mk = lambda: MLP(embed_dim, hid_dim, embed_dim, False, device, dtype, activation=activation, depth=2)  # noqa: E731
        self.mlp = nn.ModuleList([mk() for _ in range(n_mlp)])
        if layer_arch == "fmfmsm":
            self.step_kinds = [("f", 0), ("m", 0), ("f", 1), ("m", 1), ("s", 0), ("m", 2)]
        else:
            self.step_kinds = [("s", 0), ("m", 0), ("f", 0)]
        if norm_type == "rmsnorm":
            mkn = lambda: RMSNorm(embed_dim, eps=layer_norm_eps, elementwise_affine=False, device=device, dtype=dtype)  # noqa: E731
        else:
            mkn = lambda: LayerNormMixedPrecision(embed_dim, eps=layer_norm_eps, elementwise_affine=False, device=device, dtype=dtype)  # noqa: E731
        self.layer_norms = nn.ModuleList([mkn() for _ in self.step_kinds])

    @property
    def alpha(self) -> float:
        return 1.0 if self.deepnorm_alpha is None else float(self.deepnorm_alpha)

    def seq_indices(self, index=0):
        i1 = index * 2 if self.seq_attn_isolated else index
        return i1, (i1 + 1 if self.seq_attn_isolated else i1)

    # -------------------------------------------------------------- sublayers
    def run_sublayer(self, kind, idx, x, eval_pos, feature_atten_mask=None):
        if kind == "m":
            return self.mlp[idx](x)
        if kind == "f":
            mask = None
            if feature_atten_mask is not None:
                m = feature_atten_mask.bool()
                mask = (m.unsqueeze(-1) & m.unsqueeze(-2)).reshape(-1, m.shape[-1], m.shape[-1]).unsqueeze(1)
            return self.feature_attentions[idx](x, attn_mask=mask)[0]
        return self.sequence_attention(x, eval_pos, idx)

    def sequence_attention(self, x, eval_pos, index=0):
        i1, i2 = self.seq_indices(index)
        ctx = x[:, :eval_pos].transpose(1, 2)
        out_ctx = self.sequence_attentions[i1](ctx, x_kv=ctx, copy_first_head_kv=self.self_share_all_kv_heads)[0].transpose(1, 2)
        if eval_pos >= x.shape[1]:
            return out_ctx
        kv_src = out_ctx.transpose(1, 2) if self.seq_attn_serial else ctx
        out_q = self.sequence_attentions[i2](
            x[:, eval_pos:].transpose(1, 2), x_kv=kv_src, copy_first_head_kv=self.cross_share_all_kv_heads
        )[0].transpose(1, 2)
        return torch.cat([out_ctx, out_q], 1)

    def _residual(self, res, upd):
        if self.deepnorm_alpha is not None:
            return res + self.deepnorm_alpha.to(upd.dtype) * upd
        return res + upd

    def step(self, i, x, eval_pos, feature_atten_mask=None):
        kind, idx = self.step_kinds[i]
        norm = self.layer_norms[i]
        if self.pre_norm:
            return self._residual(x, self.run_sublayer(kind, idx, norm(x), eval_pos, feature_atten_mask))
        return norm(self.run_sublayer(kind, idx, x, eval_pos, feature_atten_mask) + x)

    def forward(self, x, feature_atten_mask=None, eval_pos=None, **_):
        for i in range(len(self.step_kinds)):
            x = self.step(i, x, eval_pos, feature_atten_mask)
        return x, None, None

    # -------------------------------------------------------------- KV cache
    def _cache_steps(self):
        if self.layer_arch == "fmfmsm":
            return (0, 1, 2, 3), 4, (5,)
        return (), 0, (1, 2)

    def forward_train_cache(self, x, quantize=False, row_chunk=None):
        """Run context rows through the layer and keep the cross-attention K/V."""
        from synthefy_nori_b200.models.kv_cache import QuantizedKV

        pre, s, post = self._cache_steps()
        N = x.shape[1]
        for i in pre:
            x = self.step(i, x, N)
        i1, i2 = self.seq_indices(0)
        a_self, a_cross = self.sequence_attentions[i1], self.sequence_attentions[i2]
        norm = self.layer_norms[s]
        xin = norm(x) if self.pre_norm else x
        t = xin.transpose(1, 2)
        attn = a_self(t, x_kv=t, copy_first_head_kv=self.self_share_all_kv_heads)[0].transpose(1, 2)
        src = attn if self.seq_attn_serial else xin
        cache = a_cross.project_kv_cache(src.transpose(1, 2), copy_first_head_kv=self.cross_share_all_kv_heads)
        if quantize:
            cache = QuantizedKV.from_kv(cache["kv"], cache["batch"], cache["groups"])
        x = self._residual(x, attn) if self.pre_norm else norm(attn + x)
        for i in post:
            x = self.step(i, x, N)
        return x, {"seq_kv": cache}

    def forward_test_with_cache(self, x, cache):
        pre, s, post = self._cache_steps()
        n = x.shape[1]
        for i in pre:
            x = self.step(i, x, n)
        _, i2 = self.seq_indices(0)
        norm = self.layer_norms[s]
        xin = norm(x) if self.pre_norm else x
        attn = self.sequence_attentions[i2].forward_with_kv_cache(xin.transpose(1, 2), cache["seq_kv"])[0].transpose(1, 2)
        x = self._residual(x, attn) if self.pre_norm else norm(attn + x)
        for i in post:
            x = self.step(i, x, n)
        return x


class LayerStack(nn.Module):
    def __init__(self, layers):
        super().__init__()
        self.layers = nn.ModuleList(layers)
        self.gradient_checkpointing = False

    def forward(self, x, **kw):
        for layer in self.layers:
            if self.gradient_checkpointing and self.training:
                x = checkpoint(lambda t, l=layer: l(t, **kw)[0], x, use_reentrant=False)
            else:
                x = layer(x, **kw)[0]
        return x, None, None

    def build_train_cache(self, x, quantize=False):
        caches = []
        for layer in self.layers:
            x, c = layer.forward_train_cache(x, quantize=quantize)
            caches.append(c)
        return x, caches

    def forward_test_with_cache(self, x, caches):
        if len(caches) != len(self.layers):
            raise ValueError(f"Expected {len(self.layers)} layer caches, got {len(caches)}")
        for layer, c in zip(self.layers, caches):
            x = layer.forward_test_with_cache(x, c)
        return x
