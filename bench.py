"""Headline benchmark: nori-100m DDP pretraining throughput (tables/s, whole job).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload train|train30m|infer5|infer4|infer1]

For N > 1 run under ``torch.distributed.run`` (one rank per GPU, NCCL, rendezvous on
127.0.0.1).  Headline config: nori-100m training on the pretraining table shapes:
random-init nori-100m weights, synthetic SCM-prior tables, 16 tables per GPU per step
(32, the nori-30m config's batch, does not fit the reference's nori-100m step in 180 GB),
rows ~ U[512, 2048] (one row count per step, shared by the batch), context fraction
~ U[0.5, 0.9], features ~ U[5, 100] padded to 100, 999-quantile pinball loss (+0.05
monotonicity), bf16 compute, clip 1.0, AdamW + EMA 0.999, activation checkpointing.
``--workload train30m`` is the same with nori-30m and 32 tables per GPU, the config whose
gradient exchange is largest relative to its compute (25 MB gradient buckets).

``value`` times W untimed warm-up steps then exactly K steps on the device (CUDA
events, barrier + synchronize on both sides, max over ranks); each step generates its
tables on the GPU, runs forward + backward, reduces gradients across ranks and applies
the optimizer.  Every step's activations are several GB (far above the 126 MB L2), so
no L2 flush is needed between steps.  ``e2e`` runs the same training through the
public ``NoriTrainer.train_step`` with each step's tables copied host->device from
pinned memory and the loss read back to the host.

``--impl reference`` runs the unmodified reference package from ``baseline/_ref``
(its FeaturesTransformer with bf16 autocast, SDPA attention, native RMSNorm, layer
checkpointing, the regional ``torch.compile`` of the encoder layer that its stock
launcher enables (``--reference-compile none`` for eager; a compile failure falls back
to eager and is reported), ``compute_ccmm_loss`` pinball objective, torch AdamW, its EMA
helper, DDP/NCCL with 25 MB buckets for N > 1) on the same table shapes; its tables are
generated before the timed region, and its ``e2e`` copies each step's tables from pinned
host memory and reads the loss back, like ours.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)



def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=6)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default=None, help="default: nori-100m (train), nori-30m (train30m)")
    ap.add_argument("--tables-per-gpu", type=int, default=None, help="default: 16 (train), 32 (train30m)")
    ap.add_argument("--min-rows", type=int, default=512)
    ap.add_argument("--max-rows", type=int, default=2048)
    ap.add_argument("--features", type=int, default=100)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--grad-reduction", default="peer", choices=["nccl", "peer"],
                    help="N > 1: peer = in-kernel reduce-scatter / sharded AdamW / all-gather over NVLink peer memory; "
                         "nccl = all-reduce baseline")
    ap.add_argument("--workload", default="train", choices=["train", "train30m", "infer5", "infer4", "infer1"],
                    help="train (headline: nori-100m, 16 tables/GPU), train30m (nori-30m, 32 tables/GPU, the "
                         "gradient-bound pretraining config), infer5 (256 tables x 2048 context rows, cached, "
                         "4 query calls), infer4 (one 100k-row context, int8 KV, 10k queries), infer1 (nori-6m on CPU)")
    ap.add_argument("--reference-compile", default="dynamic", choices=["dynamic", "none"],
                    help="reference arm: regional torch.compile of the encoder layer as the reference's stock "
                         "launcher enables it (dynamic), or eager (none); a compile failure falls back to eager "
                         "and is reported in the JSON line")
    ap.add_argument("--bucket-mb", type=float, default=25.0, help="peer DDP gradient bucket size (MB)")
    ap.add_argument("--profile-kernels", type=int, default=0,
                    help="after the timed region, profile one more (untimed) step on every rank and print "
                         "rank 0's top-N kernels by device time to stderr")
    ap.add_argument("--shape-palette", type=int, default=4,
                    help="number of (rows, context rows) pairs drawn once from the shape distribution and cycled over "
                         "the steps (0: a fresh shape every step); warm-up steps cover the palette, so the "
                         "reference's compiled layers run from their cache in the timed steps, as with the "
                         "reference's own --shape-palette")
    ap.add_argument("--infer-tables", type=int, default=256)
    ap.add_argument("--infer-group", type=int, default=8, help="tables per cache build / predict batch")
    args = ap.parse_args()
    if args.model is None:
        args.model = "nori-30m" if args.workload == "train30m" else "nori-100m"
    if args.tables_per_gpu is None:
        args.tables_per_gpu = 32 if args.workload == "train30m" else 16
    return args


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        self.proc = None
        self.path = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            fd, self.path = tempfile.mkstemp(prefix="nori_clocks_", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200", "-i",
                 ident], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:  # noqa: BLE001
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        loaded = [s for s in sm if s > 0.5 * smax] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": smax, "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# ----------------------------------------------------------------------------- shapes
def step_shapes(args, n: int):
    """(rows, eval_pos) of every step.  rows ~ U[min_rows, max_rows], context fraction
    ~ U[0.5, 0.9].  With a palette of P shapes, the P shapes are the distribution's
    stratum midpoints (rows and fractions at quantiles (i + 1/2) / P, fractions paired with
    rows by a seeded permutation), so the palette has the distribution's mean and mean
    square row count (attention cost grows with rows^2); the steps cycle through it."""
    g = torch.Generator().manual_seed(args.seed)
    if args.shape_palette > 0:
        P = args.shape_palette
        perm = torch.randperm(P, generator=g).tolist()
        draws = []
        for i in range(P):
            rows = int(round(args.min_rows + (i + 0.5) * (args.max_rows - args.min_rows) / P))
            frac = 0.5 + 0.4 * (perm[i] + 0.5) / P
            draws.append((rows, min(max(1, int(rows * frac)), rows - 1)))
        order = torch.randperm(P, generator=g).tolist()
        draws = [draws[i] for i in order]
        return [draws[i % P] for i in range(n)]
    out = []
    for _ in range(n):
        rows = int(torch.randint(args.min_rows, args.max_rows + 1, (1,), generator=g).item())
        frac = 0.5 + 0.4 * float(torch.rand(1, generator=g).item())
        out.append((rows, min(max(1, int(rows * frac)), rows - 1)))
    return out


def prior_cfg(args):
    from synthefy_nori_b200.training.prior import PriorConfig

    return PriorConfig(min_features=5, max_features=args.features, pad_features=args.features)


def timed(fn_steps, device, world):
    """Run fn_steps() between barriers; return max-over-ranks device milliseconds."""
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    fn_steps()
    end.record()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    ms = torch.tensor([start.elapsed_time(end)], device=device)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def count_native_launches(step_fn) -> int:
    """Kernels of this repository's extension launched by one step (profiled, untimed)."""
    from torch.profiler import ProfilerActivity, profile

    names = ("nori::", "gemm_kernel", "attn_fwd", "attn_bwd", "rms_", "pinball_kernel", "adamw_ema_kernel",
             "sumsq_kernel", "swiglu_bwd_kernel", "quant_int8_kernel", "peer_", "bucket_", "layout_sync", "qass_",
             "ln_act", "colsum", "col_stats", "rbf_aug", "assemble_", "scm_act", "scm_linear")
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    n = 0
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA and any(k in ev.name for k in names):
            n += 1
    return n


def _print_kernel_profile(step_fn, top: int, rank: int) -> None:
    """One profiled step (every rank runs it: the step has collectives); rank 0 prints the
    kernels with the most device time (all streams) to stderr."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    if rank != 0:
        return
    rows = sorted(((ev.self_device_time_total / 1000.0, ev.count, ev.key[:100]) for ev in prof.key_averages()
                   if getattr(ev, "self_device_time_total", 0) > 0), reverse=True)
    tot = sum(r[0] for r in rows)
    print(f"[profile] kernels in one step: {tot:.1f} ms (summed over streams), {sum(r[1] for r in rows)} launches",
          file=sys.stderr)
    for ms, n, k in rows[:top]:
        print(f"[profile] {ms:9.1f} ms {n:5d}  {k}", file=sys.stderr)


# ----------------------------------------------------------------------------- arms
def run_ours(args, device, world, rank):
    from synthefy_nori_b200 import ops
    from synthefy_nori_b200.models.config import preset_config
    from synthefy_nori_b200.training.prior import scm_prior_batch
    from synthefy_nori_b200.training.trainer import NoriTrainer, TrainConfig
    from synthefy_nori_b200.utils.loading import build_model

    if not ops.native_available():
        raise RuntimeError(f"native extension not loaded: {ops.native_import_error()}")
    torch.manual_seed(args.seed)
    model = build_model(preset_config(args.model))
    trainer = NoriTrainer(model, TrainConfig(grad_reduction=args.grad_reduction, bucket_mb=args.bucket_mb), device)
    pc = prior_cfg(args)
    B = args.tables_per_gpu
    shapes = step_shapes(args, args.warmup + args.steps + 1)

    def one(i):
        rows, ep = shapes[i]
        b = scm_prior_batch(pc, B, rows, ep, seed=args.seed * 1000003 + i * 7919 + rank, device=device)
        return trainer.train_step(b.x, b.y, b.eval_pos)

    for i in range(args.warmup):
        one(i)
    for i in range(args.warmup, max(args.warmup, args.shape_palette)):  # every palette shape seen once
        one(i)
    clocks = ClockSampler(device)
    losses = []
    ms = timed(lambda: [losses.append(one(args.warmup + i)) for i in range(args.steps)], device, world)
    clk = clocks.stop()
    launches = count_native_launches(lambda: one(args.warmup + args.steps)) * args.steps
    ops.check_status(device)
    e2e = None if args.no_e2e else run_e2e(args, trainer, shapes, device, world, rank)
    if args.profile_kernels > 0:
        _print_kernel_profile(lambda: one(args.warmup + args.steps), args.profile_kernels, rank)
    info = {}
    if trainer.peer is not None:
        info["grad_buckets"] = trainer.peer.describe()
        # one more (untimed) step with per-bucket CUDA events: when each bucket's reduction
        # finished relative to the end of the backward pass
        trainer.peer.record_timeline = True
        one(args.warmup + args.steps)
        torch.cuda.synchronize(device)
        rep = trainer.peer.overlap_report()
        trainer.peer.record_timeline = False
        if rep is not None:
            t = torch.tensor([rep["tail_ms"]], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            rep["tail_ms_max_over_ranks"] = round(float(t.item()), 3)
            info["grad_overlap"] = rep
    return ms, clk, launches, e2e, float(losses[-1].item()), info


def run_e2e(args, trainer, shapes, device, world, rank):
    """Public-API training from pinned host tables: H2D copy + ``NoriTrainer.train_step`` +
    ``loss.item()`` per step."""
    return _e2e_loop(args, trainer.train_step, shapes, device, world, rank)


def _compile_reference_layers(model):
    """The reference launcher's default execution speedup: one ``torch.compile`` of the
    encoder layer's forward (dynamic shapes) shared by every layer (reference
    ``training/cli.py:1371-1397``, enabled by ``scripts/train.sh:30-35``)."""
    import types

    for name in ("cache_size_limit", "recompile_limit", "accumulated_cache_size_limit",
                 "accumulated_recompile_limit"):
        if hasattr(torch._dynamo.config, name):
            setattr(torch._dynamo.config, name, 1024)
    torch._dynamo.config.optimize_ddp = False
    layers = model.transformer_encoder.layers
    compiled = torch.compile(type(layers[0]).forward, dynamic=True, fullgraph=False)
    for layer in layers:
        layer.forward = types.MethodType(compiled, layer)


def _uncompile_reference_layers(model):
    for layer in model.transformer_encoder.layers:
        layer.__dict__.pop("forward", None)


def run_reference(args, device, world, rank):
    from synthefy_nori_b200.utils.reference import import_reference

    if import_reference() is None:
        return None
    from synthefy_nori.model.layer import RMSNorm as RefRMSNorm
    from synthefy_nori.training.loss import compute_ccmm_loss
    from synthefy_nori.training.trainer import _foreach_ema_update
    from synthefy_nori.utils.loading import build_model as ref_build

    from synthefy_nori_b200.models.config import preset_config
    from synthefy_nori_b200.training.prior import scm_prior_batch

    torch.manual_seed(args.seed)
    cfg = dict(preset_config(args.model))
    cfg["mask_prediction"] = True  # the training CLI's setting (reference training/cli.py:1192)
    model = ref_build(cfg).to(device)
    for m in model.modules():  # native RMSNorm, as the training CLI enables (cli.py:1330-1342)
        if isinstance(m, RefRMSNorm):
            m.use_native = True
    model._skip_feature_decoder = True  # feature loss weight 0 (cli.py:1344-1350)
    compile_state = "none"
    if args.reference_compile == "dynamic":
        _compile_reference_layers(model)
        compile_state = "dynamic regional (encoder layer)"
    model.transformer_encoder.gradient_checkpointing = True
    model.train()
    net = model
    if world > 1:
        from torch.nn.parallel import DistributedDataParallel as DDP

        net = DDP(model, device_ids=[device.index], find_unused_parameters=False, gradient_as_bucket_view=True,
                  bucket_cap_mb=args.bucket_mb)
    params = [p for p in model.parameters() if p.requires_grad]
    opt = torch.optim.AdamW(params, lr=3e-4, betas=(0.9, 0.95), weight_decay=0.01)
    ema = {k: v.detach().clone() for k, v in model.state_dict().items()}
    quantiles = list(model.regression_quantiles)
    pc = prior_cfg(args)
    B = args.tables_per_gpu
    shapes = step_shapes(args, args.warmup + args.steps + 1)
    batches = []
    for i, (rows, ep) in enumerate(shapes[: args.warmup + args.steps]):
        b = scm_prior_batch(pc, B, rows, ep, seed=args.seed * 1000003 + i * 7919 + rank, device=device)
        batches.append((b.x, b.y, ep))

    def step(x, y, ep):
        opt.zero_grad(set_to_none=True)
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            out = net(x=x, y=y[:, :ep], eval_pos=ep, task_type="reg")
        loss, _ = compute_ccmm_loss(out, y[:, ep:], x, None, "reg", feature_loss_weight=0.0,
                                    regression_loss="pinball", regression_quantiles=quantiles,
                                    pinball_monotonicity_weight=0.05)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(params, 1.0)
        opt.step()
        _foreach_ema_update(ema, model.state_dict(), 0.999)
        return loss.detach()

    def one(i):
        return step(*batches[i])

    # warm-up; with regional compile the first shapes also compile (static, then dynamic).
    # Every rank takes the same branch: a compile failure on any rank turns compile off on all.
    failed = None
    for i in list(range(args.warmup)) + [args.warmup + j for j in range(max(0, args.shape_palette - args.warmup))]:
        try:
            one(i)
            err = 0
        except Exception as exc:  # noqa: BLE001 - Inductor / Dynamo failures surface here
            if compile_state == "none":
                raise
            failed, err = f"{type(exc).__name__}: {str(exc).splitlines()[0][:160]}", 1
        flag = torch.tensor([err], device=device)
        if world > 1:
            dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        if int(flag.item()) and compile_state != "none":
            _uncompile_reference_layers(model)
            compile_state = f"none (regional compile failed: {failed or 'on another rank'})"
            opt.zero_grad(set_to_none=True)
            torch.cuda.synchronize(device)
            one(i)
    clocks = ClockSampler(device)
    losses = []
    ms = timed(lambda: [losses.append(one(args.warmup + i)) for i in range(args.steps)], device, world)
    clk = clocks.stop()
    del batches
    e2e = None
    if not args.no_e2e:
        e2e = _e2e_loop(args, step, shapes, device, world, rank)
    return ms, clk, 0, e2e, float(losses[-1].item()), {"reference_compile": compile_state}


def _host_batches(args, shapes, device, rank):
    """Pinned host copies of the tables for the end-to-end loop (the device-timed steps'
    shapes plus one warm-up table set), generated before the timed region."""
    from synthefy_nori_b200.training.prior import scm_prior_batch

    pc = prior_cfg(args)
    host = []
    for i in range(args.steps + 1):
        rows, ep = shapes[args.warmup + i]
        b = scm_prior_batch(pc, args.tables_per_gpu, rows, ep, seed=args.seed * 7 + i + 100 * rank, device=device)
        host.append((b.x.cpu().pin_memory(), b.y.cpu().pin_memory(), ep))
    torch.cuda.synchronize(device)
    return host


def _e2e_loop(args, step, shapes, device, world, rank):
    """End to end through a step callable: every step copies its tables host->device from
    pinned memory and reads the loss back to the host inside the timed region."""
    host = _host_batches(args, shapes, device, rank)

    def one(i):
        x_h, y_h, ep = host[i]
        x = x_h.to(device, non_blocking=True)
        y = y_h.to(device, non_blocking=True)
        return float(step(x, y, ep).item())

    one(args.steps)  # warm
    ms = timed(lambda: [one(i) for i in range(args.steps)], device, world)
    h2d = sum(host[i][0].numel() * 4 + host[i][1].numel() * 4 for i in range(args.steps)) / args.steps
    tables = args.tables_per_gpu * world * args.steps
    return {"value": tables / (ms / 1000.0), "unit": "tables/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": 4, "ms_per_step": ms / args.steps}


# ----------------------------------------------------------------------------- inference
def _infer_tables(n_tables, n_ctx, n_q, n_feat, seed, device, nan_frac=0.15, n_cat=0):
    """Synthetic tables: X ~ N(0,1) (optional categorical codes), NaNs, y = random 2-layer MLP(X) + noise."""
    g = torch.Generator(device=device).manual_seed(seed)
    N = n_ctx + n_q
    X = torch.randn(n_tables, N, n_feat, generator=g, device=device)
    if n_cat:
        card = torch.randint(2, 51, (n_cat,), generator=g, device=device)
        X[:, :, :n_cat] = torch.floor(torch.rand(n_tables, N, n_cat, generator=g, device=device) * card)
    W1 = torch.randn(n_tables, n_feat, 64, generator=g, device=device) / n_feat ** 0.5
    W2 = torch.randn(n_tables, 64, 1, generator=g, device=device) / 8.0
    y = torch.bmm(torch.tanh(torch.bmm(X, W1)), W2).squeeze(-1) + 0.05 * torch.randn(n_tables, N, generator=g,
                                                                                      device=device)
    X[torch.rand(X.shape, generator=g, device=device) < nan_frac] = float("nan")
    y = (y - y[:, :n_ctx].mean(1, keepdim=True)) / y[:, :n_ctx].std(1, keepdim=True).clamp_min(1e-6)
    return X, y


def run_infer5(args, device, world, rank, impl):
    """Batched multi-table cached inference: tables data-parallel over ranks; per group of tables the context
    cache is built once, then 4 predict calls with 512 fresh query rows each (timed)."""
    n_ctx, n_feat, n_q, calls = 2048, 50, 512, 4
    per_rank = args.infer_tables // world
    grp = args.infer_group
    if impl == "reference":
        from synthefy_nori_b200.utils.reference import import_reference

        import_reference()
        from synthefy_nori.utils.loading import build_model as mk
    else:
        from synthefy_nori_b200.utils.loading import build_model as mk
    from synthefy_nori_b200.models.config import preset_config

    torch.manual_seed(args.seed)
    model = mk(dict(preset_config(args.model))).to(device).eval()
    build_ms = pred_ms = 0.0
    groups = [(i, min(grp, per_rank - i)) for i in range(0, per_rank, grp)]
    # warm-up on one group
    warm = groups[: max(1, min(args.warmup, 1))]
    for phase, gl in (("warm", warm), ("timed", groups)):
        for gi, (off, n) in enumerate(gl):
            X, y = _infer_tables(n, n_ctx, n_q * calls, n_feat, args.seed + rank * 100003 + off, device)
            if world > 1 and phase == "timed":
                dist.barrier()
            torch.cuda.synchronize(device)
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record()
            with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16, enabled=impl == "reference"):
                cache = model.build_context_cache(X[:, :n_ctx], y[:, :n_ctx], cache_dtype="bf16")
                e1.record()
                for c in range(calls):
                    xq = X[:, n_ctx + c * n_q : n_ctx + (c + 1) * n_q]
                    model.apply_context_cache(xq, cache)
            e2.record()
            torch.cuda.synchronize(device)
            if phase == "timed":
                build_ms += e0.elapsed_time(e1)
                pred_ms += e1.elapsed_time(e2)
            del cache
    t = torch.tensor([build_ms, pred_ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    build_ms, pred_ms = float(t[0]), float(t[1])
    rows = per_rank * world * n_q * calls
    return {"metric": "nori-100m batched multi-table cached inference query rows/s", "value": rows / (pred_ms / 1000),
            "unit": "query rows/s", "ms_predict_total": pred_ms, "ms_cache_build_total": build_ms,
            "tables": per_rank * world, "ctx_rows": n_ctx, "features": n_feat, "query_rows_per_call": n_q,
            "calls": calls, "group": grp}


def run_infer4(args, device, world, rank, impl):
    """Long-context inference: one table, 100k context rows x 100 features (20
    categorical), int8 KV cache, 10k query rows; build + query timed separately."""
    n_ctx = int(os.environ.get("NORI_INFER4_CTX", "100000"))
    n_q = int(os.environ.get("NORI_INFER4_QUERY", "10000"))
    from synthefy_nori_b200.models.config import preset_config

    if impl == "reference":
        from synthefy_nori_b200.utils.reference import import_reference

        import_reference()
        from synthefy_nori.utils.loading import build_model as mk
    else:
        from synthefy_nori_b200.utils.loading import build_model as mk
    torch.manual_seed(args.seed)
    model = mk(dict(preset_config(args.model))).to(device).eval()
    X, y = _infer_tables(1, n_ctx, n_q, 100, args.seed, device, nan_frac=0.10, n_cat=20)
    # warm-up (kernel attributes, tensor maps, allocator) on a small slice, untimed
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16, enabled=impl == "reference"):
        if world > 1:
            from synthefy_nori_b200.parallel.context_parallel import ShardedContextPredictor

            wsp = ShardedContextPredictor(model, device)
            wsp.build(X[:, :512], y[:, :512])
            wsp.predict_raw(X[:, n_ctx : n_ctx + 64])
            wsp.close()
        else:
            wc = model.build_context_cache(X[:, :512], y[:, :512], cache_dtype="int8")
            model.apply_context_cache(X[:, n_ctx : n_ctx + 64], wc)
            del wc
    if world > 1 and impl == "reference":
        return {"impl": "reference", "unavailable": "the reference has no multi-GPU context-sharded inference path"}
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record()
    if world > 1:
        # context rows sharded over ranks; each rank answers its slice of the queries
        from synthefy_nori_b200.parallel.context_parallel import ShardedContextPredictor

        sp = ShardedContextPredictor(model, device)
        sp.build(X[:, :n_ctx], y[:, :n_ctx])
        e1.record()
        lo, hi = rank * n_q // world, (rank + 1) * n_q // world
        for s in range(lo, hi, 2048):
            sp.predict_raw(X[:, n_ctx + s : n_ctx + min(hi, s + 2048)])
        e2.record()
        torch.cuda.synchronize(device)
        sp.close()
    else:
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16, enabled=impl == "reference"):
            cache = model.build_context_cache(X[:, :n_ctx], y[:, :n_ctx], cache_dtype="int8")
            e1.record()
            model.apply_context_cache(X[:, n_ctx:], cache, row_chunk_size=2048)
        e2.record()
        torch.cuda.synchronize(device)
    t = torch.tensor([e0.elapsed_time(e1), e1.elapsed_time(e2)], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    b, q = float(t[0]), float(t[1])
    return {"metric": "nori-100m 100k-ctx infer query rows/s", "value": n_q / ((b + q) / 1000), "unit": "query rows/s",
            "ms_cache_build": b, "ms_query": q, "ctx_rows": n_ctx, "query_rows": n_q, "cache": "int8",
            "query_rows_per_s_excluding_build": n_q / (q / 1000),
            "context_sharding": f"rows over {world} GPUs" if world > 1 else "none"}


def run_infer1(args, impl):
    """nori-6m single-table inference on the CPU (512 context rows x 10
    features, 5% NaN, y = Xw + 0.5 sin(3 x0) + N(0, 0.1^2); 128 query rows; the mean plus
    quantiles 0.1 / 0.5 / 0.9).  Wall-clock latency per call (the CPU has no device timer),
    median over the timed calls, one model forward per call (no ensemble)."""
    import numpy as np

    torch.set_num_threads(int(os.environ.get("NORI_CPU_THREADS", "8")))
    rng = np.random.default_rng(args.seed)
    X = rng.standard_normal((640, 10)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    w = rng.standard_normal(10)
    y = (np.nan_to_num(X) @ w + 0.5 * np.sin(3 * np.nan_to_num(X[:, 0])) + 0.1 * rng.standard_normal(640))
    from synthefy_nori_b200.models.config import preset_config

    if impl == "reference":
        from synthefy_nori_b200.utils.reference import import_reference

        import_reference()
        from synthefy_nori.utils.loading import build_model as mk
    else:
        from synthefy_nori_b200.utils.loading import build_model as mk
    torch.manual_seed(args.seed)
    model = mk(dict(preset_config("nori-6m"))).eval()
    taus = torch.tensor(model.regression_quantiles, dtype=torch.float64)
    xt = torch.from_numpy(X).unsqueeze(0)
    ym, ys = y[:512].mean(), y[:512].std()
    yt = torch.from_numpy(((y - ym) / ys).astype(np.float32)).unsqueeze(0)

    def call():
        with torch.no_grad():
            out = model(xt, yt[:, :512], eval_pos=512, task_type="reg")
            raw = (out["reg_output"] if isinstance(out, dict) else out)[0].double()
            q = raw.sort(-1).values
            mean = taus[0] * q[:, 0] + (1 - taus[-1]) * q[:, -1] + (0.5 * (q[:, 1:] + q[:, :-1]) * taus.diff()).sum(-1)
            idx = torch.searchsorted(taus, torch.tensor([0.1, 0.5, 0.9], dtype=torch.float64)).clamp(max=len(taus) - 1)
            return mean * ys + ym, q[:, idx] * ys + ym

    for _ in range(max(args.warmup, 1)):
        call()
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        call()
        ts.append((time.perf_counter() - t0) * 1e3)
    med = float(np.median(ts))
    return {"metric": "nori-6m single-table CPU inference latency", "value": med, "unit": "ms",
            "higher_is_better": False, "steps": args.steps, "warmup": args.warmup, "ms_all": [round(t, 2) for t in ts],
            "cpu_threads": torch.get_num_threads(), "dtype": "fp32", "data": "synthetic (config 1)",
            "config": {"model": "nori-6m", "ctx_rows": 512, "query_rows": 128, "features": 10, "device": "cpu"}}


def main_infer(args, device, world, rank):
    res = run_infer5(args, device, world, rank, args.impl) if args.workload == "infer5" else \
        run_infer4(args, device, world, rank, args.impl)
    if rank == 0 and "unavailable" in res:
        print(json.dumps(res), flush=True)
    elif rank == 0:
        res.update({"n_gpus": world, "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
                    "config": {"model": args.model, "parallelism": f"tables-dp{world}" if args.workload == "infer5"
                               else (f"context-rows-sharded-{world}" if world > 1 else "single-gpu")}})
        if args.impl == "reference":
            res["impl"] = "reference"
        print(json.dumps(res), flush=True)


def main():
    args = parse()
    if args.workload == "infer1":
        res = run_infer1(args, args.impl)
        if args.impl == "reference":
            res["impl"] = "reference"
        print(json.dumps(res), flush=True)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    t0 = time.time()
    if not args.workload.startswith("train"):
        main_infer(args, device, world, rank)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.impl == "reference":
        res = run_reference(args, device, world, rank)
        if res is None:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "reference package not installed under baseline/_ref"}))
            return
    else:
        res = run_ours(args, device, world, rank)
    ms, clk, launches, e2e, last_loss, info = res
    tables = args.tables_per_gpu * world * args.steps
    value = tables / (ms / 1000.0)
    if rank == 0:
        if world == 1:
            reduction = "none (one GPU)"
        elif args.impl == "reference":
            reduction = f"DDP/NCCL all-reduce, {args.bucket_mb:g} MB buckets"
        elif args.grad_reduction == "peer":
            reduction = f"peer-memory reduce-scatter over NVLink, {args.bucket_mb:g} MB buckets overlapped with backward"
        else:
            reduction = "NCCL all-reduce"
        line = {
            "metric": f"{args.model} train tables/s",
            "value": round(value, 3),
            "unit": "tables/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 3),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (GPU SCM-prior tables, random-init weights)",
            "config": {
                "model": args.model,
                "global_batch": args.tables_per_gpu * world,
                "seq_len": f"rows U[{args.min_rows},{args.max_rows}] x {args.features} features (padded)",
                "parallelism": f"dp{world}",
                "tables_per_gpu": args.tables_per_gpu,
                "loss": "pinball 999 + 0.05 monotonicity",
                "optimizer": "AdamW + EMA 0.999, clip 1.0",
                "l2": "per-step working set is several GB (> 126 MB L2); no flush needed",
                "shapes": (f"stratified palette of {args.shape_palette} (rows, ctx) shapes cycled"
                           if args.shape_palette > 0 else "fresh draw per step"),
            },
            "grad_reduction": reduction,
            "clocks": clk,
            "gpu_launches": launches,
            "peak_mem_gib": round(torch.cuda.max_memory_allocated(device) / 2 ** 30, 1),
            "last_loss": last_loss,
            "wall_s": round(time.time() - t0, 1),
        }
        line.update(info)
        if args.impl == "reference":
            line["impl"] = "reference"
        if e2e is not None:
            line["e2e"] = e2e
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
