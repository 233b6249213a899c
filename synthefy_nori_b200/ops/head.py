"""The regression head and the pinball objective on the native kernels.

Head (reference ``model/transformer.py:345-350``): the last token of every query row,
the encoder's output norm (LayerNorm, or an RMSNorm without weight folded into the
first GEMM as a row scale), ``Linear(E, H) -> LayerNorm(H) -> GELU -> Linear(H,
K=999)``.  ``HeadPinball`` runs it as one autograd node:

forward   out-norm (ln_act, one warp per row)  ->  tcgen05 GEMM + bias  ->  LayerNorm +
          GELU (ln_act)  ->  tcgen05 GEMM + bias (N padded to a multiple of 8)  ->
          pinball value and gradient in one pass (``pinball_fused_into``).  The logits
          are dropped as soon as the gradient is written, so only the bf16 gradient of
          the 999-wide output stays alive until the backward;
backward  dW2 (split-K weight-gradient GEMM), db2 (column sums), dG (GEMM with the
          weight read MN-major), LayerNorm + GELU backward, dW1, db1, dA, out-norm
          backward - all on this library's kernels (no cuBLAS, no eager elementwise).

The bf16 operand copies of the two weight matrices come from the trainer's persistent
layouts (refreshed by the optimizer) or, outside training, from a per-generation cast.
"""

from __future__ import annotations

import torch

from synthefy_nori_b200 import ops

BF16 = torch.bfloat16


def _pad8(n: int) -> int:
    return -(-n // 8) * 8


def head_supported(model) -> bool:
    dec = getattr(model, "reg_y_decoder", None)
    if dec is None or len(dec) != 4:
        return False
    l1, ln, act, l2 = dec
    norm = model.encoder_out_norm
    ok = (isinstance(l1, torch.nn.Linear) and isinstance(ln, torch.nn.LayerNorm) and isinstance(act, torch.nn.GELU)
          and getattr(act, "approximate", "none") == "none" and isinstance(l2, torch.nn.Linear)
          and l1.bias is not None and l2.bias is not None and ln.elementwise_affine
          and l1.in_features % 8 == 0 and l1.out_features % 8 == 0 and l1.out_features <= 2048
          and l1.in_features <= 2048)
    ok = ok and (isinstance(norm, torch.nn.Identity) or (isinstance(norm, torch.nn.LayerNorm) and norm.elementwise_affine)
                 or (_is_rms(norm) and getattr(norm, "weight", None) is None))
    return bool(ok)


def _is_rms(norm) -> bool:
    from synthefy_nori_b200.models.layers import RMSNorm

    return isinstance(norm, RMSNorm)


def head_blocks(model):
    """Weight blocks of the head for ``ops.weight_layouts``: (param, offset, rows, cols,
    key, dst offset, dst row stride) and the layout shapes (``w2`` padded to 8 rows)."""
    l1, l2 = model.reg_y_decoder[0], model.reg_y_decoder[3]
    H, Ein, K = l1.out_features, l1.in_features, l2.out_features
    blocks = [(l1.weight, 0, H, Ein, "w1", 0, Ein), (l2.weight, 0, K, H, "w2", 0, H)]
    return blocks, {"w1": (H, Ein), "w2": (_pad8(K), H)}


def _head_bf16(model) -> dict:
    dec = model.reg_y_decoder
    ptrs = tuple(p.data_ptr() for p in dec.parameters())
    pers = getattr(model, "_nori_head_layouts", None)
    if pers is not None and pers[0] == ptrs:
        return pers[1]
    from synthefy_nori_b200.ops.fused_layer import _GENERATION

    key = (_GENERATION[0], ptrs)
    hit = getattr(model, "_nori_head_cast", None)
    if hit is not None and hit[0] == key:
        return hit[1]
    l1, l2 = dec[0], dec[3]
    w2 = torch.zeros(_pad8(l2.out_features), l2.in_features, device=l2.weight.device, dtype=BF16)
    w2[: l2.out_features] = l2.weight.detach().to(BF16)
    wb = {"w1": l1.weight.detach().to(BF16).contiguous(), "w2": w2}
    model._nori_head_cast = (key, wb)
    return wb


class HeadPinball(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, norm_w, norm_b, w1, b1, ln_w, ln_b, w2, b2, target, quantiles, inv_var, cfg):
        C = ops.lib()
        nq, norm_kind, norm_eps, ln_eps, tail_w, mono_w, mse_w, wb = cfg
        R = x.shape[0]
        K = w2.shape[0]
        Kp = wb["w2"].shape[0]
        rs = None
        if norm_kind == "ln":
            a, m0, r0 = C.ln_act_fwd(x, norm_w, norm_b, norm_eps, 0)
        elif norm_kind == "rms":  # no affine weight: a row scale folded into the first GEMM
            a, m0, r0 = x.contiguous(), None, None
            rs = ops.rms_scale(a, norm_eps)
        else:
            a, m0, r0 = x, None, None
        h1 = ops.gemm(a, wb["w1"], row_scale=rs, bias=b1.detach().float().contiguous())
        g1, m1, r1 = C.ln_act_fwd(h1, ln_w, ln_b, ln_eps, 1)
        b2p = b2.detach().float()
        if Kp != K:
            b2p = torch.cat([b2p, b2p.new_zeros(Kp - K)])
        logits = ops.gemm(g1, wb["w2"], bias=b2p)
        dlog = torch.empty(R, Kp, device=x.device, dtype=BF16)
        loss = C.pinball_fused_into(logits, K, target, quantiles, inv_var, nq, tail_w, mono_w, mse_w, dlog)
        del logits
        ctx.cfg = cfg
        ctx.save_for_backward(x, a, h1, g1, dlog, norm_w, norm_b, ln_w, ln_b, w1, w2,
                              *(t for t in (m0, r0, rs) if t is not None), m1, r1)
        ctx.norm_kind = norm_kind
        return loss[0]

    @staticmethod
    def backward(ctx, gout):
        C = ops.lib()
        nq, norm_kind, norm_eps, ln_eps, tail_w, mono_w, mse_w, wb = ctx.cfg
        saved = ctx.saved_tensors
        x, a, h1, g1, dlog, norm_w, norm_b, ln_w, ln_b, w1, w2 = saved[:11]
        rs = None
        if norm_kind == "ln":
            m0, r0, m1, r1 = saved[11:]
        elif norm_kind == "rms":
            rs, m1, r1 = saved[11:]
        else:
            m1, r1 = saved[11:]
        dev = x.device
        K = w2.shape[0]
        dlog = dlog * gout.to(BF16)  # 1 / gradient-accumulation steps, or 1
        dw2 = torch.zeros(dlog.shape[1], w2.shape[1], device=dev, dtype=torch.float32)
        ops.gemm_wgrad(dlog, g1, dw2)
        db2 = torch.zeros(K, device=dev, dtype=torch.float32)
        C.colsum_bf16(dlog, db2)
        dg1 = ops.gemm(dlog, wb["w2"], w_kn=True)
        del dlog
        dh1 = torch.empty_like(h1)
        dln_w = torch.zeros_like(ln_w, dtype=torch.float32)
        dln_b = torch.zeros_like(ln_b, dtype=torch.float32)
        C.ln_act_bwd(dg1, h1, ln_w.detach().float(), ln_b.detach().float(), m1, r1, 1, dh1, dln_w, dln_b)
        dw1 = torch.zeros_like(w1, dtype=torch.float32)
        ops.gemm_wgrad(dh1, ops.rms_apply(a, rs) if rs is not None else a, dw1)
        db1 = torch.zeros(w1.shape[0], device=dev, dtype=torch.float32)
        C.colsum_bf16(dh1, db1)
        da = ops.gemm(dh1, wb["w1"], w_kn=True)
        dnw = dnb = None
        if norm_kind == "ln":
            dx = torch.empty(x.shape, device=dev, dtype=BF16)
            dnw = torch.zeros_like(norm_w, dtype=torch.float32)
            dnb = torch.zeros_like(norm_b, dtype=torch.float32)
            C.ln_act_bwd(da, x, norm_w.detach().float(), norm_b.detach().float(), m0, r0, 0, dx, dnw, dnb)
        elif norm_kind == "rms":
            dx = ops.rms_bwd(da, a, rs)
        else:
            dx = da
        return (dx, dnw, dnb, dw1, db1, dln_w, dln_b, dw2[:K], db2, None, None, None, None)


def head_pinball_loss(model, last_tokens: torch.Tensor, target: torch.Tensor, quantiles: torch.Tensor,
                      tail_weight: float = 0.0, monotonicity_weight: float = 0.0, mse_weight: float = 0.0):
    """Pinball objective of the regression head on ``last_tokens`` ``[B * nq, E]`` (bf16,
    rows may be strided) against ``target [B, nq]``; the same value as
    ``training.loss.pinball_objective(model.reg_y_decoder(model.encoder_out_norm(.)))``."""
    B, nq = target.shape
    l1, ln, _, l2 = model.reg_y_decoder
    norm = model.encoder_out_norm
    has_norm = isinstance(norm, torch.nn.LayerNorm)
    kind = "ln" if has_norm else ("rms" if _is_rms(norm) else "none")
    t = target.float()
    inv_var = (1.0 / t.var(dim=1, unbiased=False).clamp(min=0.01)).contiguous()
    wb = _head_bf16(model)
    cfg = (nq, kind, float(norm.eps) if kind != "none" else None, float(ln.eps), float(tail_weight),
           float(monotonicity_weight), float(mse_weight), wb)
    nw = norm.weight if has_norm else None
    nb = norm.bias if has_norm else None
    return HeadPinball.apply(last_tokens, nw, nb, l1.weight, l1.bias, ln.weight, ln.bias, l2.weight, l2.bias,
                             t.reshape(-1).contiguous(), quantiles.float().contiguous(), inv_var, cfg)
