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


def _dp_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import numpy as np

        from synthefy_nori_b200.inference.predictor import NoriPredictor
        from synthefy_nori_b200.models.config import preset_config
        from synthefy_nori_b200.parallel.distributed_inference import DistributedInference, table_parallel_predict
        from synthefy_nori_b200.utils.loading import build_model

        torch.manual_seed(0)
        model = build_model(preset_config("nori-tiny")).eval()
        rng = np.random.default_rng(0)
        X = rng.standard_normal((47, 4)).astype(np.float32)
        y = X[:, 0].copy()
        pred = NoriPredictor(model, "cpu", n_estimators=1)
        ctx = pred.fit_context(X[:30], y[:30])
        full = pred.predict_raw(ctx, X[30:])
        got = DistributedInference(pred).predict_raw(ctx, torch.from_numpy(X[30:]))
        q.put((rank, "query", float((got - full).abs().max())))
        xt = torch.from_numpy(rng.standard_normal((3, 40, 4)).astype(np.float32))
        yt = xt[..., 0].clone()
        ref = model.apply_context_cache(xt[:, 30:], model.build_context_cache(xt[:, :30], yt[:, :30])).float()
        tp = table_parallel_predict(model, xt[:, :30], yt[:, :30], xt[:, 30:])
        q.put((rank, "tables", float((tp - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_distributed_inference_on_gloo():
    import socket

    world = 2
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_dp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(2 * world)]
    for p in ps:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in ps)
    assert all(v < 1e-5 for _, _, v in res), res


def _leave_worker(rank, world, port, q):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    from synthefy_nori_b200.parallel.health import RankFailure, RankHealth

    store = dist.distributed_c10d._get_default_store()
    health = RankHealth(store, rank, world, stale_s=30.0)
    g = torch.ones(4)
    health.beat(0)
    dist.all_reduce(g)  # step 0 on both ranks
    dist.barrier()
    if rank == 1:
        health.leave()  # leaves between steps, with nothing in flight
        q.put((rank, "left", None))
        q.close()
        q.join_thread()  # flush the queue before the hard exit
        os._exit(0)  # no destroy_process_group: the process just ends
    import time

    time.sleep(1.0)
    t0 = time.time()
    try:
        health.check(1)
        q.put((rank, "check", "no error"))
    except RankFailure as e:
        q.put((rank, "check", e.ranks))
    t1 = time.time()
    try:
        dist.all_reduce(g)  # the next collective ends with an error, within the group timeout
        q.put((rank, "collective", "no error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "collective", type(e).__name__))
    q.put((rank, "times", (t1 - t0, time.time() - t1)))
    q.close()
    q.join_thread()
    os._exit(0)


@pytest.mark.timeout(120)
def test_rank_leaving_between_steps_is_detected():
    import socket

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_leave_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = {}
    for _ in range(4):
        r, k, v = q.get(timeout=90)
        got[(r, k)] = v
    for p in ps:
        p.join(timeout=30)
    assert got[(0, "check")] == [1]  # the host-side check names the rank that left
    assert got[(0, "collective")] != "no error"
    t_check, t_coll = got[(0, "times")]
    assert t_check < 2.0 and t_coll < 30.0


def test_rank_health_staleness():
    from synthefy_nori_b200.parallel.health import RankFailure, RankHealth

    class Store(dict):
        def set(self, k, v):
            self[k] = v.encode() if isinstance(v, str) else v

        def get(self, k):
            return dict.__getitem__(self, k)

        def check(self, keys):
            return all(k in self for k in keys)

    st = Store()
    a, b = RankHealth(st, 0, 2, stale_s=60.0, max_lag=2), RankHealth(st, 1, 2, stale_s=60.0, max_lag=2)
    a.beat(5)
    b.beat(5)
    a.check(6)
    with pytest.raises(RankFailure) as e:
        a.check(9)  # rank 1 is 4 steps behind
    assert e.value.ranks == [1]
    st["nori/health/1"] = b"5 0.0"  # a heartbeat from long ago
    with pytest.raises(RankFailure):
        a.check(5)
