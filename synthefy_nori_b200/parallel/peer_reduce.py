"""Data-parallel optimizer step over NVLink peer memory (no NCCL on the step path).

``PeerDDP`` owns IPC-shareable flat fp32 parameter / gradient buffers (model parameters
and their ``.grad`` become views into them), exchanges the CUDA IPC handles once through
the process group, and runs one fused peer step per optimizer step:
flag -> per-shard gradient reduction by P2P loads + norm partials -> clip + AdamW + EMA
on the owned shard (sharded optimizer state) -> all-gather of the updated shards by P2P
loads. See ``csrc/peer.cu``.  The NCCL baseline is ``dist.all_reduce`` of the same flat
gradient buffer followed by the replicated fused AdamW step (``training/optim.py``).
"""

from __future__ import annotations

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


def exchange_handles(local: dict, group=None) -> list[dict]:
    """All-gather small per-rank dicts (IPC handles as bytes) over the process group."""
    world = dist.get_world_size(group)
    out: list = [None] * world
    dist.all_gather_object(out, local, group=group)
    return out


class PeerDDP:
    def __init__(self, params, device: torch.device, group=None, lr=3e-4, betas=(0.9, 0.95), eps=1e-8,
                 weight_decay=0.01, ema_decay=0.999, max_grad_norm=1.0, align: int = 64):
        from synthefy_nori_b200 import ops

        C = ops.lib()
        self.C = C
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("PeerDDP supports up to 8 ranks (one NVLink domain)")
        self.device = device
        self.params = [p for p in params if p.requires_grad]
        self.offsets, off = [], 0
        for p in self.params:
            self.offsets.append(off)
            off += -(-p.numel() // align) * align
        self.numel = off
        W = self.world
        # local IPC-shareable buffers
        self._own = {
            "param": C.peer_malloc(self.numel * 4),
            "grad": C.peer_malloc(self.numel * 4),
            "flags": C.peer_malloc(3 * W * 8),
            "norms": C.peer_malloc(W * 4),
        }
        dev = device.index
        self.data = C.tensor_from_ptr(self._own["param"], self.numel, dev, torch.float32)
        self.grad = C.tensor_from_ptr(self._own["grad"], self.numel, dev, torch.float32)
        for p, o in zip(self.params, self.offsets):
            n = p.numel()
            self.data[o : o + n].copy_(p.detach().reshape(-1).to(self.data))
            p.data = self.data[o : o + n].view(p.shape)
            p.grad = self.grad[o : o + n].view(p.shape)
        torch.cuda.synchronize(device)
        handles = {k: bytes(C.peer_ipc_handle(v).numpy().tobytes()) for k, v in self._own.items()}
        allh = exchange_handles(handles, group)
        self._opened = []
        self.ptrs = {k: [] for k in self._own}
        for r, h in enumerate(allh):
            for k in self._own:
                if r == self.rank:
                    self.ptrs[k].append(self._own[k])
                else:
                    ptr = C.peer_ipc_open(torch.frombuffer(bytearray(h[k]), dtype=torch.uint8))
                    self._opened.append(ptr)
                    self.ptrs[k].append(ptr)
        b = shard_bounds(self.numel, W, 4)
        self.bounds = torch.tensor(b, dtype=torch.int64, device=device)
        self.s0, self.s1 = b[self.rank], b[self.rank + 1]
        n = self.s1 - self.s0
        self.red = torch.zeros(max(n, 1), device=device)
        self.m = torch.zeros(max(n, 1), device=device)
        self.v = torch.zeros(max(n, 1), device=device)
        self.ema = self.data[self.s0 : self.s1].clone() if ema_decay is not None else None
        self.local_norm = torch.zeros(1, device=device)
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.ema_decay, self.max_grad_norm = ema_decay, max_grad_norm
        self.step_count = 0
        self.flag_step = 0
        dist.barrier(group)

    def zero_grad(self) -> None:
        self.grad.zero_()

    def step(self) -> None:
        """Reduce gradients across ranks (mean), clip, AdamW + EMA on the owned shard,
        all-gather parameters. Stream-ordered; no host synchronisation."""
        from synthefy_nori_b200.ops.api import status_word

        self.step_count += 1
        self.flag_step += 1
        self.C.peer_ddp_step(self.ptrs["grad"], self.ptrs["param"], self.ptrs["flags"], self.ptrs["norms"], self.rank,
                             self.s0, self.s1, self.bounds, self.flag_step, self.red, self.m, self.v, self.ema,
                             self.local_norm, self.lr, self.betas[0], self.betas[1], self.eps, self.wd,
                             self.step_count, self.ema_decay if self.ema_decay is not None else 0.0,
                             self.max_grad_norm or 0.0, 1.0 / self.world, status_word(self.device))

    def gather_ema(self) -> torch.Tensor | None:
        """Full EMA vector (all shards), gathered with the process group."""
        if self.ema is None:
            return None
        b = self.bounds.tolist()
        width = max(b[i + 1] - b[i] for i in range(self.world))
        buf = torch.zeros(width, device=self.device)
        buf[: self.s1 - self.s0] = self.ema
        parts = [torch.empty_like(buf) for _ in range(self.world)]
        dist.all_gather(parts, buf, group=self.group)
        return torch.cat([parts[i][: b[i + 1] - b[i]] for i in range(self.world)])

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        for p in self._opened:
            self.C.peer_ipc_close(p)
        self._opened = []
        dist.barrier(self.group)
        for v in self._own.values():
            self.C.peer_free(v)
        self._own = {}
