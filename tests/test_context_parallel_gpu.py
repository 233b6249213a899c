"""Context-row-sharded inference (int8 K/V shards in peer memory; query attention over
staged, dequantised shards on the tcgen05 kernel with LSE merges, and over the shards
read in place by the multi-shard int8 kernel) against the single-GPU int8 context cache,
on 2 and 4 GPUs (skipped with fewer)."""

import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _run(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from synthefy_nori_b200.models.config import preset_config
        from synthefy_nori_b200.parallel.context_parallel import ShardedContextPredictor
        from synthefy_nori_b200.utils.loading import build_model

        torch.manual_seed(0)
        model = build_model(preset_config("nori-tiny")).to(dev).eval()
        g = torch.Generator(device=dev).manual_seed(3)
        x = torch.randn(1, 700, 9, generator=g, device=dev)
        y = torch.randn(1, 600, generator=g, device=dev)
        sp = ShardedContextPredictor(model, dev)
        sp.build(x[:, :600], y)
        nq = 100
        lo, hi = rank * nq // world, (rank + 1) * nq // world
        part = sp.predict_raw(x[:, 600 + lo : 600 + hi]).float().cpu()
        sp.query_attention = "q8_shards"
        part_q8 = sp.predict_raw(x[:, 600 + lo : 600 + hi]).float().cpu()
        sp.close()
        ref = None
        if rank == 0:
            with torch.no_grad():
                cache = model.build_context_cache(x[:, :600], y, cache_dtype="int8")
                ref = model.apply_context_cache(x[:, 600:], cache).float().cpu()
        from synthefy_nori_b200 import ops

        ops.check_status(dev)
        q.put((rank, part, ref, part_q8))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 4])
def test_sharded_context_matches_single_gpu_cache(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29100 + (os.getpid() % 500) + 11 * world
    procs = [ctx.Process(target=_run, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=240) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = res[0][2]
    for k in (1, 3):  # staged tcgen05 path, in-place multi-shard int8 kernel
        got = torch.cat([r[k] for r in res], 1)
        assert got.shape == ref.shape
        cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
        assert cos > 0.999, cos
        assert (got - ref).abs().max().item() < 0.05 * ref.abs().max().item() + 0.02
