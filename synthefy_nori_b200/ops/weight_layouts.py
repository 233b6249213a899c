"""Persistent bf16 operand layouts of the native encoder layers.

The native layer (and the native regression head) reads its weights as bf16 GEMM
operands in fused layouts: the
context-row projection ``[Wqkv_self; Wkv_cross]`` (5 x H x Dp rows, Dp = the head width
rounded up to 8 with zero rows), the query projection,
the two sequence output projections and the feature output projection in their stored
``[E_in, E_out]`` form (read MN-major by the GEMM), the SwiGLU gate/up rows
interleaved, the down projection and the feature QKV projection.

For training, the fp32 master weights live in one flat buffer (``FlatParams`` or the
peer-memory ``PeerDDP`` buffer), and ``WeightLayouts`` keeps one bf16 tensor per
layout, refreshed after every optimizer step by ONE kernel launch (``layout_sync``)
that walks a segment table: segment = a row-major block of the flat buffer written to a
strided block of one layout.  With several ranks the same kernel is the parameter
all-gather: it reads each element from the rank that owns it (peer memory), writes it
into the local fp32 master buffer and into the bf16 layout in the same pass.

Without a flat buffer (inference), ``fused_layer._cached_bf16`` casts the layouts once
per weight generation instead.
"""

from __future__ import annotations

import torch

from synthefy_nori_b200 import ops

CHUNK = 16384  # elements per work item of the sync kernel (a multiple of 4)


def _layer_blocks(layer):
    """(parameter, element offset in it, rows, cols, layout key, dst element offset, dst row
    stride).  Head-major weights (``[k, H, D, E]`` projections, ``[H, D, E]`` output
    projections) are written with each head's D rows at a pitch of Dp rows (D rounded up
    to 8): one block per (k, head) when D is not a multiple of 8, so the padded rows stay
    zero."""
    E = layer.embed_dim
    sa_self, sa_cross = layer.sequence_attentions[0], layer.sequence_attentions[1]
    mlp = layer.mlp[0]
    fa = layer.feature_attentions[0]
    gelu = layer.activation != "swiglu"
    hd = (mlp.mlp[0].weight if gelu else mlp.w_gate.weight).shape[0]
    H = sa_self.num_heads
    D = E // H
    Dp = -(-D // 8) * 8
    A = H * Dp

    def heads(p, k0, nk, key, dst_row0, shared=False):
        """``nk`` head-major slabs of ``p`` starting at slab ``k0`` -> layout rows from
        ``dst_row0`` at the padded pitch; with ``shared`` (MQA K/V) every head's rows are
        copied from head 0."""
        if Dp == D and not shared:
            return [(p, k0 * H * D * E, nk * H * D, E, key, dst_row0 * E, E)]
        return [(p, ((k0 + k) * H + (0 if shared else h)) * D * E, D, E, key, (dst_row0 + k * A + h * Dp) * E, E)
                for k in range(nk) for h in range(H)]

    return (
        heads(sa_self.qkv_proj_weight, 0, 1, "w_ctx", 0)
        + heads(sa_self.qkv_proj_weight, 1, 2, "w_ctx", A, shared=layer.self_share_all_kv_heads)
        + heads(sa_cross.qkv_proj_weight, 1, 2, "w_ctx", 3 * A, shared=layer.cross_share_all_kv_heads)
        + heads(sa_cross.qkv_proj_weight, 0, 1, "w_q", 0)
        + heads(sa_self.out_proj_weight, 0, 1, "wo_self", 0)
        + heads(sa_cross.out_proj_weight, 0, 1, "wo_cross", 0)
        + ([  # GELU MLP: the first projection as stored, no interleave
            (mlp.mlp[0].weight, 0, hd, E, "w_gu", 0, E),
            (mlp.mlp[-1].weight, 0, E, hd, "w_down", 0, hd),
        ] if gelu else [
            (mlp.w_gate.weight, 0, hd, E, "w_gu", 0, 2 * E),
            (mlp.w_up.weight, 0, hd, E, "w_gu", E, 2 * E),
            (mlp.w_down.weight, 0, E, hd, "w_down", 0, hd),
        ])
        + heads(fa.qkv_proj_weight, 0, 3, "w_fqkv", 0)
        + heads(fa.out_proj_weight, 0, 1, "w_fo", 0)
    )


def layout_shapes(layer) -> dict:
    E = layer.embed_dim
    H = layer.sequence_attentions[0].num_heads
    A = H * (-(-(E // H) // 8) * 8)
    gelu = layer.activation != "swiglu"
    hd = (layer.mlp[0].mlp[0].weight if gelu else layer.mlp[0].w_gate.weight).shape[0]
    return {"w_ctx": (5 * A, E), "w_q": (A, E), "wo_self": (A, E), "wo_cross": (A, E),
            "w_gu": (hd if gelu else 2 * hd, E),
            "w_down": (E, hd), "w_fqkv": (3 * A, E), "w_fo": (A, E)}


def _uncovered(ranges, numel: int) -> list:
    """Element ranges ``[(offset, length)]`` of a parameter that no block in ``ranges`` reads."""
    gaps, pos = [], 0
    for off, n in sorted(ranges):
        if off > pos:
            gaps.append((pos, off - pos))
        pos = max(pos, off + n)
    if pos < numel:
        gaps.append((pos, numel - pos))
    return gaps


def segment_plan(model, offsets: dict, with_gather: bool):
    """Pure planning step (no device work): ``(segments, chunks, layouts)`` where each
    segment is ``(src_flat_offset, rows, cols, (layer_index, key) | None, dst_offset,
    dst_row_stride)``, each chunk ``(segment, j0, j1)``, and ``layouts`` maps layer index
    to ``{key: shape}``.  ``offsets`` maps ``id(param)`` to the parameter's flat offset.
    With ``with_gather`` every trainable parameter is covered exactly once (plain
    segments without a layout for the parameters no layout reads)."""
    from synthefy_nori_b200.ops.fused_layer import layer_supported

    segs, layouts, covered = [], {}, {}
    for li, layer in enumerate(model.transformer_encoder.layers):
        if not layer_supported(layer):
            continue
        layouts[li] = layout_shapes(layer)
        for p, off, rows, cols, key, doff, drs in _layer_blocks(layer):
            if id(p) not in offsets:
                raise ValueError("a native layer weight is not in the flat parameter buffer")
            if cols % 4 or drs % 4 or doff % 4 or off % 4:
                raise ValueError("layout blocks must be 4-element aligned")
            segs.append((offsets[id(p)] + off, rows, cols, (li, key), doff, drs))
            covered.setdefault(id(p), set()).add((off, rows * cols))
    from synthefy_nori_b200.ops.head import head_blocks, head_supported

    if head_supported(model) and all(id(p) in offsets for p in model.reg_y_decoder.parameters()):
        blocks, shapes = head_blocks(model)
        layouts["head"] = shapes
        for p, off, rows, cols, key, doff, drs in blocks:
            segs.append((offsets[id(p)] + off, rows, cols, ("head", key), doff, drs))
            covered.setdefault(id(p), set()).add((off, rows * cols))
    if with_gather:
        for p in model.parameters():
            if not p.requires_grad or id(p) not in offsets:
                continue
            gaps = _uncovered(covered.get(id(p), set()), p.numel())
            for off, n in gaps:  # elements no layout reads (a whole parameter, or MQA's unused heads)
                if off % 4:
                    raise ValueError("layout blocks must be 4-element aligned")
                n4 = -(-n // 4) * 4 if off + n == p.numel() else n  # flat buffers pad each parameter
                segs.append((offsets[id(p)] + off, 1, n4, None, 0, 0))
    chunks = []
    for si, (_, rows, cols, *_rest) in enumerate(segs):
        total = rows * cols
        for j0 in range(0, total, CHUNK):
            chunks.append((si, j0, min(total, j0 + CHUNK)))
    return segs, chunks, layouts


class WeightLayouts:
    """bf16 layouts of every native layer of ``model``, kept in sync with a flat fp32
    parameter buffer (``offsets``: ``id(param) -> flat offset``)."""

    def __init__(self, model, offsets: dict, device: torch.device, with_gather: bool = False):
        segs, chunks, shapes = segment_plan(model, offsets, with_gather)
        self.device = device
        self.tensors = {}
        layers = model.transformer_encoder.layers
        for li, sh in shapes.items():
            # zeros: padded rows (the head's output width rounded up to 8) stay zero
            self.tensors[li] = {k: torch.zeros(s, device=device, dtype=torch.bfloat16) for k, s in sh.items()}
        rows = []
        for src, r, c, dst, doff, drs in segs:
            addr = 0
            if dst is not None:
                t = self.tensors[dst[0]][dst[1]]
                addr = t.data_ptr() + 2 * doff
            rows.append((src, r, c, addr, drs))
        self.seg = torch.tensor(rows, dtype=torch.int64, device=device).view(-1, 5)
        self.chunks = torch.tensor(chunks, dtype=torch.int64, device=device).view(-1, 3)
        self.n_segments = len(rows)
        for li, t in self.tensors.items():
            if li == "head":
                model._nori_head_layouts = (tuple(p.data_ptr() for p in model.reg_y_decoder.parameters()), t)
            else:
                layers[li]._nori_layouts = (tuple(p.data_ptr() for p in layers[li].parameters()), t)

    def sync(self, param_ptrs: list[int], rank: int = 0, bstart=None, bper=None) -> None:
        """Refresh every layout from the flat buffers (one launch on the current stream);
        with bucket geometry, also gather each element from the rank that owns it."""
        ops.lib().layout_sync(self.seg, self.chunks, [int(p) for p in param_ptrs], int(rank), bstart, bper,
                              ops.status_word(self.device))

    @staticmethod
    def detach(model) -> None:
        for layer in model.transformer_encoder.layers:
            if hasattr(layer, "_nori_layouts"):
                del layer._nori_layouts
        if hasattr(model, "_nori_head_layouts"):
            del model._nori_head_layouts
