"""Data-parallel optimizer step over NVLink peer memory, overlapped with the backward pass
(no NCCL on the step path).

``PeerDDP`` re-homes the trainable parameters into one IPC-shareable flat fp32 buffer,
laid out in reverse registration order (the order the backward pass produces
gradients), and cuts it into buckets of ``bucket_mb``.  Every bucket is split into
``world`` pieces; rank r owns piece r of every bucket (its reduced gradient, AdamW
moments and EMA: sharded optimizer state, 1/world of the memory).

Per optimizer step (all device work stream-ordered, no host synchronisation):

* during ``loss.backward()``, a post-accumulate-grad hook counts each bucket's
  parameters; buckets are released in index order: when bucket b and every bucket
  before it have all their gradients queued on the compute stream, a send stream (after
  an event wait) casts the bucket to the bf16 wire buffer and flags it to every peer,
  and a reduce stream waits (bounded) for the peers' flags and reduces this rank's piece
  with P2P loads (bf16 -> fp32, x 1/world, sum of squares for the clip) - so the
  reduce-scatter of bucket b overlaps the backward of the layers before it.  Sends never
  wait on peers, so no ordering between ranks can deadlock the two streams;
* ``finish()`` after the backward: norm partials and step-status bits exchanged, clip +
  AdamW + EMA on the owned pieces, then the all-gather kernel reads every peer's
  updated pieces into the local fp32 buffer and the bf16 operand layouts of the native
  layers in one pass (``ops.weight_layouts``); the compute stream waits on the comm
  stream before the next forward.

Gradient accumulation: micro-steps before the last run with ``sync=False`` (no hooks
fire, gradients accumulate locally), as DDP's ``no_sync``.

Reference: DDP with ``gradient_as_bucket_view`` and 25 MB buckets (training/cli.py:
1446-1452), no-sync accumulation (training/trainer.py:1500-1512), clip + AdamW + EMA
(trainer.py:1544-1552).
"""

from __future__ import annotations

import weakref

import torch
import torch.distributed as dist


def shard_bounds(numel: int, world: int, align: int = 4) -> list[int]:
    """Split [0, numel) into ``world`` contiguous shards whose starts are ``align``-aligned."""
    if world < 1:
        raise ValueError("world must be >= 1")
    per = -(-numel // world)
    per = -(-per // align) * align
    b = [min(i * per, numel) for i in range(world)] + [numel]
    return b


def plan_buckets(sizes: list[int], bucket_elems: int, world: int, align: int = 64):
    """Flat layout of parameters (given in bucket order) and their buckets.

    Returns ``(offsets, numel, buckets)``: every parameter starts on an ``align``
    boundary; a bucket is ``(start, end, piece)`` with ``end - start`` the padded size of
    whole parameters (at least one), ``piece`` the ``align``-rounded size of each rank's
    share (rank r owns ``[start + r piece, min(start + (r+1) piece, end))``)."""
    offsets, off = [], 0
    for n in sizes:
        offsets.append(off)
        off += -(-n // align) * align
    buckets, b0, cur = [], 0, 0
    for i, n in enumerate(sizes):
        cur = offsets[i] + -(-n // align) * align
        if cur - b0 >= bucket_elems or i == len(sizes) - 1:
            buckets.append((b0, cur))
            b0 = cur
    out = []
    for s, e in buckets:
        piece = -(-(e - s) // world)
        piece = max(align, -(-piece // align) * align)
        out.append((s, e, piece))
    return offsets, off, out


def owned_pieces(buckets, world: int, rank: int):
    """``[(red_offset, flat_offset, length)]`` of rank ``rank``'s pieces, in bucket order."""
    tab, roff = [], 0
    for s, e, piece in buckets:
        a = min(s + rank * piece, e)
        b = min(s + (rank + 1) * piece, e)
        tab.append((roff, a, b - a))
        roff += b - a
    return tab, roff


def exchange_handles(local: dict, group=None) -> list[dict]:
    """All-gather small per-rank dicts (IPC handles as bytes) over the process group."""
    world = dist.get_world_size(group)
    out: list = [None] * world
    dist.all_gather_object(out, local, group=group)
    return out


class PeerDDP:
    def __init__(self, model, device: torch.device, group=None, lr=3e-4, betas=(0.9, 0.95), eps=1e-8,
                 weight_decay=0.01, ema_decay=0.999, max_grad_norm=1.0, bucket_mb: float = 25.0,
                 wire: str = "bf16", wait_limit_s: float = 60.0, align: int = 64, record_timeline: bool = False,
                 sm_reserve: int = 4):
        from synthefy_nori_b200 import ops
        from synthefy_nori_b200.ops.weight_layouts import WeightLayouts

        if wire not in ("bf16", "fp32"):
            raise ValueError("wire must be 'bf16' or 'fp32'")
        C = ops.lib()
        self.C = C
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("PeerDDP supports up to 8 ranks (one NVLink domain)")
        self.device = device
        self.wire_bf16 = wire == "bf16"
        self.wait_limit_s = float(wait_limit_s)
        # the bucket kernels (flag wait, pack, reduce) run on side streams during the
        # backward; the persistent compute kernels leave `sm_reserve` SMs to them, so neither
        # side waits for an SM the other holds (a flag wait can last until the peer catches up)
        self.sm_reserve = int(sm_reserve) if self.world > 1 else 0
        self._prev_reserve = C.sm_reserve()
        C.set_sm_reserve(max(self._prev_reserve, self.sm_reserve))
        self.reduce_ctas = 2 * self.sm_reserve if self.sm_reserve > 0 else 64
        self.params = [p for p in model.parameters() if p.requires_grad]
        order = list(reversed(self.params))  # the backward pass produces gradients roughly in this order
        offs, self.numel, self.buckets = plan_buckets([p.numel() for p in order], int(bucket_mb * 2 ** 20 / 4),
                                                       self.world, align)
        self.offsets = [0] * len(self.params)
        pos = {id(p): i for i, p in enumerate(self.params)}
        for p, o in zip(order, offs):
            self.offsets[pos[id(p)]] = o
        W, nb = self.world, len(self.buckets)
        self.nb = nb
        own = {"param": C.peer_malloc(self.numel * 4), "flags": C.peer_malloc((nb + 2) * W * 8),
               "xchg": C.peer_malloc(2 * W * 4)}
        if self.wire_bf16:
            own["wire"] = C.peer_malloc(self.numel * 2)
            self.grad = torch.zeros(self.numel, device=device)
        else:
            own["wire"] = C.peer_malloc(self.numel * 4)  # the gradient buffer itself is read by peers
        self._own = own
        dev = device.index
        self.data = C.tensor_from_ptr(own["param"], self.numel, dev, torch.float32)
        if not self.wire_bf16:
            self.grad = C.tensor_from_ptr(own["wire"], self.numel, dev, torch.float32)
        for p, o in zip(self.params, self.offsets):
            n = p.numel()
            self.data[o : o + n].copy_(p.detach().reshape(-1).to(self.data))
            p.data = self.data[o : o + n].view(p.shape)
            p.grad = self.grad[o : o + n].view(p.shape)
        torch.cuda.synchronize(device)
        handles = {k: bytes(C.peer_ipc_handle(v).numpy().tobytes()) for k, v in own.items()}
        allh = exchange_handles(handles, group)
        self._opened = []
        self.ptrs = {k: [] for k in own}
        for r, h in enumerate(allh):
            for k in own:
                if r == self.rank:
                    self.ptrs[k].append(own[k])
                else:
                    ptr = C.peer_ipc_open(torch.frombuffer(bytearray(h[k]), dtype=torch.uint8))
                    self._opened.append(ptr)
                    self.ptrs[k].append(ptr)
        # bucket of every parameter; pieces owned by this rank
        self.bucket_of = {}
        starts = [s for s, _, _ in self.buckets]
        import bisect

        for p, o in zip(self.params, self.offsets):
            self.bucket_of[id(p)] = bisect.bisect_right(starts, o) - 1
        # Parameters expected to receive a gradient every step: all of them until the first
        # synchronised step has shown which ones do (task-specific heads stay unused); a
        # bucket is released once its expected parameters are done.
        self.expected = None
        self._fired: set = set()
        self._stale = False
        self.bucket_count = [0] * nb
        for b in self.bucket_of.values():
            self.bucket_count[b] += 1
        tab, n_owned = owned_pieces(self.buckets, W, self.rank)
        self.pieces = tab
        self.max_piece = max((t[2] for t in tab), default=0)
        self.piece_tab = torch.tensor(tab, dtype=torch.int64, device=device).view(-1, 3)
        self.bstart = torch.tensor(starts + [self.buckets[-1][1] if nb else 0], dtype=torch.int64, device=device)
        self.bper = torch.tensor([pc for _, _, pc in self.buckets], dtype=torch.int64, device=device)
        self.red = torch.zeros(max(n_owned, 4), device=device)
        self.m = torch.zeros(max(n_owned, 4), device=device)
        self.v = torch.zeros(max(n_owned, 4), device=device)
        self.ema = self.owned_from_full(self.data) if ema_decay is not None else None
        self.norm_acc = torch.zeros(1, device=device)
        self.bits = torch.zeros(1, device=device)
        self.diag = torch.zeros(2, device=device)
        self.counters = torch.zeros(max(nb, 1), dtype=torch.int32, device=device)
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.ema_decay, self.max_grad_norm = ema_decay, max_grad_norm
        self.step_count = 0
        self.flag_step = 0
        self.comm = torch.cuda.Stream(device)  # waits + reductions + optimizer + all-gather
        self.send = torch.cuda.Stream(device)  # bucket pack + signal (never waits on a peer)
        self.record_timeline = record_timeline
        self.timeline: list = []
        self._remaining = list(self.bucket_count)
        self._launched = [False] * nb
        self._next = 0
        self._sync = False
        self._active = False
        offsets_by_id = {id(p): o for p, o in zip(self.params, self.offsets)}
        self.layouts = WeightLayouts(model, offsets_by_id, device, with_gather=True)
        self.layouts.sync([own["param"]])  # initial bf16 layouts from the local (broadcast) weights
        self._hooks = [p.register_post_accumulate_grad_hook(self._hook) for p in self.params]
        model._nori_layout_owner = weakref.ref(self)
        self._model = model
        torch.cuda.synchronize(device)
        dist.barrier(group)

    # ------------------------------------------------------------------ geometry helpers
    def owned_from_full(self, full: torch.Tensor) -> torch.Tensor:
        """This rank's pieces of a full flat vector, concatenated."""
        parts = [full[f : f + n] for _, f, n in self.pieces]
        out = torch.cat(parts) if parts else full.new_zeros(0)
        return out if out.numel() >= 4 else torch.cat([out, out.new_zeros(4 - out.numel())])

    def full_from_owned(self, owned: torch.Tensor) -> torch.Tensor:
        """Full flat vector assembled from every rank's pieces (collective over the group)."""
        W = self.world
        sizes = [owned_pieces(self.buckets, W, r)[1] for r in range(W)]
        width = max(max(sizes), 4)
        buf = torch.zeros(width, device=self.device)
        buf[: sizes[self.rank]] = owned[: sizes[self.rank]]
        parts = [torch.empty_like(buf) for _ in range(W)]
        dist.all_gather(parts, buf, group=self.group)
        full = torch.zeros(self.numel, device=self.device)
        for r in range(W):
            tab, _ = owned_pieces(self.buckets, W, r)
            for roff, f, n in tab:
                full[f : f + n] = parts[r][roff : roff + n]
        return full

    def describe(self) -> dict:
        return {"buckets": self.nb, "bucket_mb": round(max((e - s) for s, e, _ in self.buckets) * 4 / 2 ** 20, 2)
                if self.nb else 0, "wire": "bf16" if self.wire_bf16 else "fp32", "params": len(self.params),
                "numel": self.numel}

    # ------------------------------------------------------------------ step protocol
    def zero_grad(self) -> None:
        self.grad.zero_()

    def begin(self, sync: bool = True) -> None:
        """Start a micro-step; ``sync`` marks the last micro-step of an optimizer step
        (its backward reduces gradients bucket by bucket)."""
        self._sync = sync
        if sync:
            self.flag_step += 1
            self._fired = set()
            self._stale = False
            self._remaining = list(self.bucket_count)
            self._launched = [False] * self.nb
            self._next = 0
            self._active = True
            cur = torch.cuda.current_stream(self.device)
            self.comm.wait_stream(cur)
            self.send.wait_stream(cur)
            with torch.cuda.stream(self.comm):
                self.norm_acc.zero_()
            if self.record_timeline:
                self.timeline = []

    def _hook(self, p) -> None:
        if not self._sync:
            return
        b = self.bucket_of[id(p)]
        self._fired.add(id(p))
        if self.expected is not None and id(p) not in self.expected:
            # a parameter that had no gradient in the first step has one now: fine while its
            # bucket is still open; if the bucket was already sent, finish() redoes the round
            if self._launched[b]:
                self._stale = True
            return
        self._remaining[b] -= 1
        # release buckets in index order (the same order on every rank)
        while self._next < self.nb and self._remaining[self._next] == 0:
            self._launch(self._next)
            self._next += 1

    def _launch(self, b: int) -> None:
        if self._launched[b]:
            return
        self._launched[b] = True
        from synthefy_nori_b200 import ops

        s, e, _ = self.buckets[b]
        W, rank = self.world, self.rank
        ready = torch.cuda.Event(enable_timing=self.record_timeline)
        ready.record(torch.cuda.current_stream(self.device))
        self.send.wait_event(ready)
        st = ops.status_word(self.device)
        with torch.cuda.stream(self.send):
            self.C.peer_bucket_pack_signal(self.grad.data_ptr(), self.ptrs["wire"][rank] if self.wire_bf16 else 0,
                                           s, e - s, self.counters.data_ptr() + 4 * b, self.ptrs["flags"], rank, b * W,
                                           self.flag_step, self.device.index)
        with torch.cuda.stream(self.comm):
            ev0 = None
            if self.record_timeline:
                ev0 = torch.cuda.Event(enable_timing=True)
                ev0.record(self.comm)
            self.C.peer_wait(self.ptrs["flags"][rank], b * W, W, self.flag_step, self.wait_limit_s, st)
            roff, f0, n = self.pieces[b]
            self.C.peer_bucket_reduce(self.ptrs["wire"], f0, n, self.wire_bf16, 1.0 / W,
                                      self.red.data_ptr() + 4 * roff, self.norm_acc.data_ptr(), st,
                                      self.reduce_ctas)
            if self.record_timeline:
                ev1 = torch.cuda.Event(enable_timing=True)
                ev1.record(self.comm)
                self.timeline.append((b, ready, ev0, ev1))

    def finish(self, bits: torch.Tensor | None = None) -> None:
        """After the backward of the last micro-step: reduce any bucket not yet launched
        (parameters without a gradient this step), exchange norms and status, clip +
        AdamW + EMA on the owned pieces, all-gather into fp32 master + bf16 layouts."""
        from synthefy_nori_b200 import ops

        if not self._active:
            raise RuntimeError("PeerDDP.finish() without begin(sync=True)")
        end_bwd = None
        if self.record_timeline:
            end_bwd = torch.cuda.Event(enable_timing=True)
            end_bwd.record(torch.cuda.current_stream(self.device))
            self.timeline.append(("backward_end", end_bwd, None, None))
        for b in range(self._next, self.nb):  # buckets with a parameter that got no gradient
            self._launch(b)
        self._next = self.nb
        if self._stale:
            # every rank runs the same graph, so every rank takes this branch: send and
            # reduce every bucket again under a new flag generation
            self.flag_step += 1
            self._launched = [False] * self.nb
            with torch.cuda.stream(self.comm):
                self.norm_acc.zero_()
            for b in range(self.nb):
                self._launch(b)
        if self.expected is None or self._stale:
            self.expected = set(self._fired) | (self.expected or set())
            self.bucket_count = [0] * self.nb
            for p in self.params:
                if id(p) in self.expected:
                    self.bucket_count[self.bucket_of[id(p)]] += 1
        self._active = False
        self._sync = False
        self.step_count += 1
        W, rank, nb = self.world, self.rank, self.nb
        st = ops.status_word(self.device)
        cur = torch.cuda.current_stream(self.device)
        if bits is not None:
            self.bits.copy_(bits.reshape(1).float())
        else:
            self.bits.zero_()
        self.comm.wait_stream(cur)
        with torch.cuda.stream(self.comm):
            self.C.peer_publish(self.ptrs["flags"], self.ptrs["xchg"], rank, self.norm_acc.data_ptr(),
                                self.bits.data_ptr(), nb * W, self.flag_step)
            self.C.peer_wait(self.ptrs["flags"][rank], nb * W, W, self.flag_step, self.wait_limit_s, st)
            self.C.peer_adamw(self.ptrs["param"], self.ptrs["xchg"], rank, self.piece_tab, self.red, self.m, self.v,
                              self.ema, self.lr, self.betas[0], self.betas[1], self.eps, self.wd, self.step_count,
                              self.ema_decay if self.ema_decay is not None else 0.0, self.max_grad_norm or 0.0,
                              self.max_piece, self.diag, st)
            self.C.peer_signal(self.ptrs["flags"], rank, nb * W + W, self.flag_step)
            self.C.peer_wait(self.ptrs["flags"][rank], nb * W + W, W, self.flag_step, self.wait_limit_s, st)
            self.layouts.sync(self.ptrs["param"], rank, self.bstart, self.bper)
            if self.record_timeline:
                end = torch.cuda.Event(enable_timing=True)
                end.record(self.comm)
                self.timeline.append(("finish", None, None, end))
        cur.wait_stream(self.comm)
        cur.wait_stream(self.send)

    def overlap_report(self) -> dict | None:
        """From the last step recorded with ``record_timeline`` (after a synchronize):
        per-bucket reduce end relative to the end of the backward pass (negative = the
        bucket was reduced while the backward was still running) and the time from the
        end of the backward to the end of the step's communication."""
        if not self.timeline:
            return None
        end_bwd = next((t[1] for t in self.timeline if t[0] == "backward_end"), None)
        fin = next((t[3] for t in self.timeline if t[0] == "finish"), None)
        if end_bwd is None or fin is None:
            return None
        rows = [(b, ev1) for b, _, _, ev1 in self.timeline if isinstance(b, int)]
        rel = [end_bwd.elapsed_time(ev1) for _, ev1 in rows]
        return {"buckets": len(rows), "reduced_before_backward_end": sum(1 for r in rel if r < 0),
                "bucket_reduce_end_ms_rel_backward_end": [round(r, 3) for r in rel],
                "tail_ms": round(end_bwd.elapsed_time(fin), 3)}

    def resync_layouts(self) -> None:
        """Refresh the bf16 layouts from the local fp32 buffer (after weights were loaded)."""
        self.layouts.sync([self._own["param"]])

    def gather_ema(self) -> torch.Tensor | None:
        """Full EMA vector (all pieces), gathered with the process group."""
        if self.ema is None:
            return None
        return self.full_from_owned(self.ema)

    def close(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []
        if self.C.sm_reserve() == max(self._prev_reserve, self.sm_reserve):
            self.C.set_sm_reserve(self._prev_reserve)
        ref = getattr(self._model, "_nori_layout_owner", None)
        if ref is not None and ref() is self:
            del self._model._nori_layout_owner
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        for p in self._opened:
            self.C.peer_ipc_close(p)
        self._opened = []
        dist.barrier(self.group)
        # parameters keep working after close: move them off the IPC buffer
        keep = self.data.clone()
        for p, o in zip(self.params, self.offsets):
            p.data = keep[o : o + p.numel()].view(p.shape)
            p.grad = None
        from synthefy_nori_b200.ops.weight_layouts import WeightLayouts

        WeightLayouts.detach(self._model)
        from synthefy_nori_b200.ops.fused_layer import bump_weight_generation

        bump_weight_generation()
        for v in self._own.values():
            self.C.peer_free(v)
        self._own = {}
