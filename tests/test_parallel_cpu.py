"""Host-side logic of the data-parallel paths on CPU ranks (gloo, world size 2)."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from synthefy_nori_b200.parallel.peer_reduce import exchange_handles, shard_bounds


def test_shard_bounds_cover_and_align():
    for numel in (0, 1, 7, 64, 1000, 99_662_708):
        for world in (1, 2, 3, 8):
            b = shard_bounds(numel, world)
            assert b[0] == 0 and b[-1] == numel and len(b) == world + 1
            assert all(b[i] <= b[i + 1] for i in range(world))
            assert all(x % 4 == 0 for x in b[:-1] if x < numel)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        got = exchange_handles({"grad": bytes([rank] * 64), "rank": rank})
        q.put((rank, [g["rank"] for g in got], [g["grad"][0] for g in got]))
        # the DDP fallback: all-reduce of one flat gradient buffer, averaged
        g = torch.full((10,), float(rank + 1))
        dist.all_reduce(g)
        q.put((rank, "mean", float(g[0]) / world))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_handle_exchange_and_flat_allreduce_on_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=60) for _ in range(2 * world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ex = [r for r in res if r[1] != "mean"]
    for rank, ranks, first in ex:
        assert ranks == [0, 1] and first == [0, 1]
    means = [r[2] for r in res if r[1] == "mean"]
    assert means == [1.5, 1.5]
