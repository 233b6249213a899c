"""Peer-memory data-parallel step (IPC buffers, P2P reduce / sharded AdamW / all-gather)
against the NCCL all-reduce step, on 2 GPUs (skipped with fewer)."""

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
        from synthefy_nori_b200.training.prior import PriorConfig, scm_prior_batch
        from synthefy_nori_b200.training.trainer import NoriTrainer, TrainConfig
        from synthefy_nori_b200.utils.loading import build_model

        out = {}
        for mode in ("nccl", "peer"):
            torch.manual_seed(0)
            tr = NoriTrainer(build_model(preset_config("nori-tiny")), TrainConfig(grad_reduction=mode, lr=1e-3), dev)
            for step in range(3):
                b = scm_prior_batch(PriorConfig(max_features=10, pad_features=10), 2, 96, 64, seed=10 * step + rank,
                                    device=dev)
                tr.train_step(b.x, b.y, b.eval_pos)
            torch.cuda.synchronize(dev)
            out[mode] = torch.cat([p.detach().reshape(-1).float().cpu() for p in tr.model.parameters()])
            tr.close()
        from synthefy_nori_b200 import ops

        ops.check_status(dev)
        q.put((rank, out["nccl"], out["peer"]))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 4])
def test_peer_step_matches_nccl_step(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + (os.getpid() % 500) + 11 * world
    procs = [ctx.Process(target=_run, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=240) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # ranks agree, and the peer path matches the NCCL path
    for r in res[1:]:  # every rank holds identical weights
        torch.testing.assert_close(res[0][1], r[1], atol=0, rtol=0)
        torch.testing.assert_close(res[0][2], r[2], atol=0, rtol=0)
    torch.testing.assert_close(res[0][2], res[0][1], atol=1e-5, rtol=1e-4)
