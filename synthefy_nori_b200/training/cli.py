"""Pretraining entry point: ``python -m synthefy_nori_b200.training.cli`` (or under
``torchrun`` for data-parallel training on one node).

Mirrors the reference CLI's contract (``training/cli.py:423-1641``, ``trainer.py``):
a named architecture (or explicit dimensions), synthetic SCM-prior tables generated on
the GPU each step with one shape per step shared by all ranks (shared RNG) and per-rank
table seeds, pinball-999 loss with a monotonicity term, AdamW + EMA with clip 1.0, a
warmup-constant-decay learning-rate schedule (trainer.py:66-84), periodic atomic
checkpoints (temp file + ``os.replace``, trainer.py:1776-1789) and exact resume: model,
optimizer moments, EMA, step counter and RNG state are restored, so 2 + 2 resumed steps
equal 4 uninterrupted ones.

Checkpoint format: ``{"model_config", "model_state_dict", "ema_state_dict",
"optimizer_state", "step", "training_config", "rng_state"}`` - the ``model_config`` +
weights pair loads with ``utils.loading.load_model`` like a released checkpoint.
"""

from __future__ import annotations

import argparse
import dataclasses
import datetime
import json
import math
import os
import sys
import time

import torch
import torch.distributed as dist


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description="Nori pretraining on synthetic tables (B200 native)")
    g = ap.add_argument_group("architecture")
    g.add_argument("--model", default="nori-6m", help="architecture preset")
    g.add_argument("--embed-dim", type=int)
    g.add_argument("--hid-dim", type=int)
    g.add_argument("--nhead", type=int)
    g.add_argument("--nlayers", type=int)
    g.add_argument("--mask-prediction", action="store_true", help="add the masked-cell reconstruction objective")
    g.add_argument("--feature-loss-weight", type=float, default=0.5)
    g = ap.add_argument_group("schedule")
    g.add_argument("--total-steps", type=int, default=1000)
    g.add_argument("--run-steps", type=int, default=None, help="stop after this many steps in this invocation")
    g.add_argument("--batch-size", type=int, default=16, help="tables per GPU per micro-step")
    g.add_argument("--gradient-accumulation", type=int, default=1, help="micro-steps per optimizer step")
    g.add_argument("--lr", type=float, default=3e-4)
    g.add_argument("--weight-decay", type=float, default=0.01)
    g.add_argument("--betas", type=float, nargs=2, default=(0.9, 0.95))
    g.add_argument("--eps", type=float, default=1e-8)
    g.add_argument("--max-grad-norm", type=float, default=1.0)
    g.add_argument("--warmup-steps", type=int, default=100)
    g.add_argument("--decay-start-step", type=int, default=None, help="default: 80%% of total steps")
    g.add_argument("--min-lr-ratio", type=float, default=0.0)
    g.add_argument("--ema-decay", type=float, default=0.999)
    g = ap.add_argument_group("objective and optimizer")
    g.add_argument("--loss", default="pinball", choices=["pinball", "mse", "smooth_l1", "huber", "bar_distribution"])
    g.add_argument("--pinball-monotonicity-weight", type=float, default=0.05)
    g.add_argument("--pinball-tail-weight", type=float, default=0.0)
    g.add_argument("--pinball-mse-weight", type=float, default=0.0)
    g.add_argument("--num-bars", type=int, default=0)
    g.add_argument("--bar-soft-sigma", type=float, default=None)
    g.add_argument("--optimizer", default="adamw", choices=["adamw", "muon"])
    g.add_argument("--muon-include-nd", action="store_true")
    g.add_argument("--muon-include-embeddings", action="store_true")
    g.add_argument("--loss-spike-factor", type=float, default=10.0, help="skip steps above this x loss EMA (0: off)")
    g.add_argument("--loss-spike-warmup", type=int, default=50)
    g.add_argument("--no-checkpoint-layers", action="store_true", help="keep every layer's activations")
    g = ap.add_argument_group("data-parallel gradient path")
    g.add_argument("--grad-reduction", default="peer", choices=["peer", "nccl"])
    g.add_argument("--bucket-mb", type=float, default=25.0)
    g.add_argument("--grad-wire", default="bf16", choices=["bf16", "fp32"])
    g.add_argument("--peer-wait-s", type=float, default=60.0)
    g.add_argument("--heartbeat-stale-s", type=float, default=0.0,
                   help="> 0: ranks exchange heartbeats and stop when a peer goes stale or leaves")
    g = ap.add_argument_group("table shapes")
    g.add_argument("--min-rows", type=int, default=256)
    g.add_argument("--max-rows", type=int, default=1024)
    g.add_argument("--min-features", type=int, default=5)
    g.add_argument("--max-features", type=int, default=100)
    g.add_argument("--max-budget", type=int, default=10 ** 9, help="rows x features cap per table")
    g.add_argument("--dim-bias-samples", type=float, default=1.0, help="> 1 biases the row draw toward the maximum")
    g.add_argument("--dim-bias-features", type=float, default=1.0)
    g.add_argument("--context-ratio-min", type=float, default=0.5)
    g.add_argument("--context-ratio-max", type=float, default=0.9)
    g.add_argument("--shape-buckets", action="store_true", help="snap shapes to the bucket grid")
    g.add_argument("--shape-palette", default="", help="rows:features:weight,... (explicit shapes)")
    g.add_argument("--context-ratio-palette", default="", help="comma-separated context ratios")
    g.add_argument("--fixed-size", default="", help="rows,features (one fixed shape)")
    g = ap.add_argument_group("synthetic prior")
    g.add_argument("--prior", default="simple", choices=["simple", "scm", "mixture"],
                   help="simple: the random-MLP SCM of the benchmark; scm: meta-sampled MLP / tree SCMs; "
                        "mixture: all generator families")
    for fam, default in (("scm", 0.34), ("tree", 0.08), ("gp", 0.12), ("quadratic-surface", 0.06),
                         ("sparse-nonlinear", 0.08), ("lookup", 0.04), ("cat-dominant", 0.08), ("binary", 0.04),
                         ("temporal", 0.10), ("clean-lowdim", 0.06)):
        name = f"--{fam}-prob" if fam in ("cat-dominant", "clean-lowdim", "sparse-nonlinear", "quadratic-surface") \
            else f"--{fam}-prior-prob"
        g.add_argument(name, type=float, default=default)
    g.add_argument("--augment", action="store_true", help="feature-shape, categorical, heavy-tail and missingness "
                                                          "augmentations (mixture prior)")
    g.add_argument("--prefetch-workers", type=int, default=0, help="> 0: generate batches on the host in workers")
    g.add_argument("--icl-filter-model", default=None, help="checkpoint (or hub name) of a frozen filter model")
    g.add_argument("--icl-filter-reg-min-r2", type=float, default=0.05)
    g.add_argument("--icl-filter-max-rounds", type=int, default=6)
    g.add_argument("--learnability-filter", action="store_true",
                   help="keep a table only if small tree ensembles fitted on its context rows score on its queries")
    g.add_argument("--learnability-filter-reg-min-score", type=float, default=0.10)
    g.add_argument("--icl-scaling-filter", action="store_true",
                   help="keep a table only if more context rows improve the tree ensembles' query score")
    g.add_argument("--icl-scaling-min-improvement", type=float, default=0.03)
    g = ap.add_argument_group("checkpoints and logging")
    g.add_argument("--checkpoint-dir", default=None)
    g.add_argument("--save-interval", type=int, default=1000)
    g.add_argument("--resume", default=None, help="checkpoint file to resume from ('latest' = checkpoint-dir)")
    g.add_argument("--init-from", default=None, help="start from a checkpoint's weights only (fresh optimizer)")
    g.add_argument("--log-interval", type=int, default=10)
    g.add_argument("--diagnostics-interval", type=int, default=0, help="> 0: component gradient norms and phase "
                                                                         "timings every N steps")
    g.add_argument("--metrics-file", default=None, help="append one JSON line per log record")
    g.add_argument("--wandb-project", default=None)
    g.add_argument("--wandb-name", default=None)
    g.add_argument("--seed", type=int, default=0)
    _add_reference_flags(ap)
    args = ap.parse_args(argv)
    args.notices = _apply_reference_flags(args)
    return args


def _quantile_list(text: str) -> list:
    qs = [float(v) for v in text.split(",") if v.strip()]
    if not qs or any(not 0.0 < q < 1.0 for q in qs):
        raise argparse.ArgumentTypeError("quantiles must be a comma-separated list in (0, 1)")
    return qs


def _add_reference_flags(ap) -> None:
    """The reference launcher's flag names (``training/cli.py:424-1092`` of the reference),
    so its launch scripts' command lines run here. Each maps onto a setting of this CLI or of
    the model config; flags for machinery this build replaces (torch.compile, PyTorch's
    RMSNorm / foreach EMA, autocast) are accepted and reported as not applying."""
    g = ap.add_argument_group("reference launcher flags (mapped onto the settings above)")
    g.add_argument("--regression-loss", default=None, choices=["mse", "smooth_l1", "huber", "pinball",
                                                               "bar_distribution"], help="= --loss")
    g.add_argument("--regression-quantiles", type=_quantile_list, default=None,
                   help="comma-separated pinball quantiles (default: the 999-level grid)")
    g.add_argument("--bar-borders-low", type=float, default=None, help="bar_distribution: lowest border (context std)")
    g.add_argument("--bar-borders-high", type=float, default=None)
    g.add_argument("--min-samples", type=int, default=None, help="= --min-rows")
    g.add_argument("--max-samples", type=int, default=None, help="= --max-rows")
    g.add_argument("--feature-positional-embedding-type", default=None, choices=["subortho", "learned", "none"])
    g.add_argument("--feature-positional-embedding-num-slots", type=int, default=None)
    g.add_argument("--column-specific-y-aware", action="store_true", help="column-specific target-aware gating")
    g.add_argument("--no-target-aware-embedding", action="store_true")
    g.add_argument("--no-qassmax", action="store_true", help="plain softmax in the sequence attention")
    g.add_argument("--model-v2-lite", action="store_true", help="SwiGLU + RMSNorm + pre-norm / DeepNorm (the presets)")
    g.add_argument("--checkpoint", default=None, help="model_config from a checkpoint (.pt / .ckpt) or JSON file")
    g.add_argument("--resume-model-only", action="store_true", help="with --resume: weights only (= --init-from)")
    g.add_argument("--gradient-checkpointing", action="store_true", help="layer checkpointing (the default here)")
    g.add_argument("--task-type", default="reg", choices=["both", "cls", "reg"], help="this build trains 'reg'")
    g.add_argument("--regression-only", action="store_true", help="regression episodes only (always, here)")
    g.add_argument("--no-prefetch", action="store_true", help="= --prefetch-workers 0")
    g.add_argument("--prefetch-count", type=int, default=None, help="host prefetch workers (= --prefetch-workers)")
    g.add_argument("--context-missingness-prob", type=float, default=None,
                   help="> 0: missing-cell augmentation with this probability (turns --augment on)")
    g.add_argument("--heavy-tail-prior-prob", type=float, default=None,
                   help="> 0: heavy-tailed column augmentation with this probability (turns --augment on)")
    g.add_argument("--device", default=None, help="single-process runs: the CUDA device (default cuda:LOCAL_RANK)")
    g.add_argument("--no-wandb", action="store_true")
    g.add_argument("--wandb-entity", default=None)
    g.add_argument("--wandb-group", default=None)
    g.add_argument("--wandb-job-type", default=None)
    g.add_argument("--wandb-tags", default=None, help="comma-separated")
    for flag in ("--compile", "--compile-pinball-loss", "--compile-encoder-layers", "--compile-disable-ddp-optimizer",
                 "--native-rms-norm", "--ema-foreach", "--no-mixed-precision"):
        g.add_argument(flag, action="store_true", help="accepted; replaced here by the native kernels")
    g.add_argument("--compile-mode", default=None, help="accepted; replaced here by the native kernels")
    g.add_argument("--compile-cache-limit", type=int, default=None, help="accepted; replaced here by the native kernels")


def _apply_reference_flags(args) -> list[str]:
    """Fold the reference-named flags into this CLI's settings; returns notices to print."""
    notes = []
    if args.task_type != "reg":
        raise SystemExit(f"--task-type {args.task_type}: this build trains regression only (use --task-type reg)")
    if args.regression_loss is not None:
        args.loss = args.regression_loss
    if args.min_samples is not None:
        args.min_rows = args.min_samples
    if args.max_samples is not None:
        args.max_rows = args.max_samples
    if args.no_prefetch:
        args.prefetch_workers = 0
    elif args.prefetch_count is not None:
        args.prefetch_workers = args.prefetch_count
    if args.resume_model_only:
        if not args.resume:
            raise SystemExit("--resume-model-only needs --resume")
        args.init_from, args.resume = args.resume, None
    probs = {k: v for k, v in (("missing_prob", args.context_missingness_prob),
                               ("heavy_prob", args.heavy_tail_prior_prob)) if v is not None}
    if any(v > 0.0 for v in probs.values()):
        if args.prior != "mixture":
            notes.append("missing-cell / heavy-tail augmentation applies to the mixture prior (--prior mixture)")
        args.augment = probs  # augment_table probabilities (the others keep their defaults)
    if args.no_wandb:
        args.wandb_project = None
    replaced = [f for f in ("compile", "compile_pinball_loss", "compile_encoder_layers", "compile_disable_ddp_optimizer",
                            "native_rms_norm", "ema_foreach") if getattr(args, f)]
    if replaced or args.compile_mode or args.compile_cache_limit:
        notes.append("compile / native-RMSNorm / foreach-EMA flags do not apply: the encoder, loss and optimizer "
                     "already run as fused sm_100a kernels")
    if args.no_mixed_precision:
        notes.append("--no-mixed-precision does not apply: the native path computes in bf16 with fp32 accumulation "
                     "and fp32 master weights")
    return notes


def _family_probs(args) -> dict:
    return {"scm": args.scm_prior_prob, "tree": args.tree_prior_prob, "gp": args.gp_prior_prob,
            "quadratic": args.quadratic_surface_prob, "sparse_nonlinear": args.sparse_nonlinear_prob,
            "lookup": args.lookup_prior_prob, "cat_dominant": args.cat_dominant_prob, "binary": args.binary_prior_prob,
            "temporal": args.temporal_prior_prob, "clean_lowdim": args.clean_lowdim_prob}


def _shape_config(args, fpg: int):
    from synthefy_nori_b200.training.shapes import ShapeConfig

    palette = [tuple(float(v) if i == 2 else int(v) for i, v in enumerate(e.split(":")))
               for e in args.shape_palette.split(",") if e]
    ratios = [float(v) for v in args.context_ratio_palette.split(",") if v]
    fixed = tuple(int(v) for v in args.fixed_size.split(",")) if args.fixed_size else None
    return ShapeConfig(min_samples=args.min_rows, max_samples=args.max_rows, min_features=args.min_features,
                       max_features=args.max_features, features_per_group=fpg, max_budget=args.max_budget,
                       dim_bias_samples=args.dim_bias_samples, dim_bias_features=args.dim_bias_features,
                       context_ratio_min=args.context_ratio_min, context_ratio_max=args.context_ratio_max,
                       bucketed=args.shape_buckets, shape_palette=palette, context_ratio_palette=ratios, fixed=fixed)


def make_tables(prior: str, batch: int, rows: int, features: int, eval_pos: int, seed: int, device, family_probs=None,
                augment: bool = False):
    """One micro-batch ``(x [B, rows, features], y [B, rows])`` of the chosen prior."""
    import torch as _t

    if prior == "simple":
        from synthefy_nori_b200.training.prior import PriorConfig, scm_prior_batch

        lo = min(5, features)
        b = scm_prior_batch(PriorConfig(min_features=lo, max_features=features, pad_features=features), batch, rows,
                            eval_pos, seed=seed, device=_t.device(device))
        return b.x, b.y
    if prior == "scm":
        import numpy as _np

        from synthefy_nori_b200.training.scm_prior import scm_prior_tables

        rng = _np.random.default_rng(seed)
        nf = [int(rng.integers(min(2, features), features + 1)) for _ in range(batch)]
        x, y, _ = scm_prior_tables(batch, rows, nf, eval_pos, seed, _t.device(device), pad_features=features)
        return x, y
    from synthefy_nori_b200.training.generators import generate_batch

    x, y, _, _ = generate_batch(batch, rows, eval_pos, seed, _t.device(device), min_features=min(2, features),
                                max_features=features, pad_features=features, family_probs=family_probs,
                                augment=augment)
    return x, y


def _host_batch(spec, seed):
    """Prefetch-worker entry: ``spec`` = (prior, batch, shape config, family probs, augment, rank, base seed)."""
    from synthefy_nori_b200.training.shapes import ShapeSampler

    prior, batch, shape_cfg, fam, augment, rank, base = spec
    sampler = ShapeSampler(shape_cfg, base + seed)  # the step's shape: the same on every rank
    rows, feats, ratio = sampler.sample()
    ep = ShapeSampler.eval_pos(rows, ratio)
    x, y = make_tables(prior, batch, rows, feats, ep, (base * 1_000_003 + seed * 9973 + rank) & 0x7FFFFFFF, "cpu",
                       fam, augment)
    return x, y, ep


def wcd_lr(step: int, base: float, warmup: int, decay_start: int, total: int, min_ratio: float) -> float:
    """Warmup (linear) - constant - decay (cosine to ``min_ratio * base``)."""
    if step < warmup:
        return base * (step + 1) / max(warmup, 1)
    if step < decay_start:
        return base
    frac = (step - decay_start) / max(total - decay_start, 1)
    frac = min(max(frac, 0.0), 1.0)
    return base * (min_ratio + (1.0 - min_ratio) * 0.5 * (1.0 + math.cos(math.pi * frac)))


def _model_config(args) -> dict:
    from synthefy_nori_b200.models.config import apply_v2_lite, finalize_arch_config, preset_config, set_dims

    if getattr(args, "checkpoint", None):
        if args.checkpoint.endswith(".json"):
            with open(args.checkpoint) as f:
                cfg = json.load(f)
        else:
            cfg = dict(torch.load(args.checkpoint, map_location="cpu", weights_only=False)["model_config"])
    else:
        cfg = preset_config(args.model)
    if getattr(args, "model_v2_lite", False):
        apply_v2_lite(cfg)
    if getattr(args, "feature_positional_embedding_type", None) is not None:
        cfg["feature_positional_embedding_type"] = args.feature_positional_embedding_type
    if getattr(args, "feature_positional_embedding_num_slots", None) is not None:
        cfg["feature_positional_embedding_num_slots"] = args.feature_positional_embedding_num_slots
    if getattr(args, "column_specific_y_aware", False):
        cfg["use_column_specific_y_aware"] = True
    if getattr(args, "no_target_aware_embedding", False):
        cfg["use_target_aware_embedding"] = False
    if getattr(args, "no_qassmax", False):
        cfg["use_qassmax"] = False
        cfg.pop("qass_mode", None)
    dec = cfg.setdefault("decoder_config", {})
    for src, key in (("bar_borders_low", "bar_borders_low"), ("bar_borders_high", "bar_borders_high")):
        if getattr(args, src, None) is not None:
            dec[key] = float(getattr(args, src))
    if getattr(args, "regression_quantiles", None) is not None and getattr(args, "loss", "pinball") == "pinball":
        from synthefy_nori_b200.models.config import set_regression_head

        set_regression_head(cfg, quantiles=args.regression_quantiles)
    if any(v is not None for v in (args.embed_dim, args.hid_dim, args.nhead, args.nlayers)):
        set_dims(cfg, embed_dim=args.embed_dim, hid_dim=args.hid_dim, nhead=args.nhead, nlayers=args.nlayers)
        apply_v2_lite(cfg)
        finalize_arch_config(cfg)
    if getattr(args, "loss", "pinball") in ("mse", "smooth_l1", "huber"):
        from synthefy_nori_b200.models.config import set_regression_head

        set_regression_head(cfg, loss=args.loss)  # point losses train a one-output head
    return cfg


def _atomic_save(obj, path: str) -> None:
    tmp = f"{path}.tmp{os.getpid()}"
    torch.save(obj, tmp)
    os.replace(tmp, path)


class Run:
    def __init__(self, args, device, rank, world):
        from synthefy_nori_b200.training.shapes import ShapeSampler
        from synthefy_nori_b200.training.trainer import NoriTrainer, TrainConfig
        from synthefy_nori_b200.utils.loading import build_model

        self.args, self.device, self.rank, self.world = args, device, rank, world
        self.model_config = _model_config(args)
        if args.mask_prediction:
            self.model_config["mask_prediction"] = True
        torch.manual_seed(args.seed)
        model = build_model(dict(self.model_config))
        if args.init_from:
            from synthefy_nori_b200.utils.loading import load_state_into

            load_state_into(model, args.init_from)
        self.tcfg = TrainConfig(lr=args.lr, weight_decay=args.weight_decay, betas=tuple(args.betas), eps=args.eps,
                                ema_decay=args.ema_decay, max_grad_norm=args.max_grad_norm,
                                pinball_tail_weight=args.pinball_tail_weight,
                                pinball_monotonicity_weight=args.pinball_monotonicity_weight,
                                pinball_mse_weight=args.pinball_mse_weight,
                                checkpoint_layers=not args.no_checkpoint_layers, grad_reduction=args.grad_reduction,
                                bucket_mb=args.bucket_mb, grad_wire=args.grad_wire, peer_wait_s=args.peer_wait_s,
                                gradient_accumulation=args.gradient_accumulation, optimizer=args.optimizer,
                                muon_include_nd=args.muon_include_nd,
                                muon_include_embeddings=args.muon_include_embeddings, loss=args.loss,
                                num_bars=args.num_bars, bar_soft_sigma=args.bar_soft_sigma,
                                loss_spike_factor=args.loss_spike_factor or None,
                                loss_spike_warmup=args.loss_spike_warmup, mask_prediction=args.mask_prediction,
                                feature_loss_weight=args.feature_loss_weight)
        self.trainer = NoriTrainer(model, self.tcfg, device)
        self.shape_cfg = _shape_config(args, model.features_per_group)
        self.shapes = ShapeSampler(self.shape_cfg, args.seed + 17)  # shared across ranks
        self.family_probs = _family_probs(args)
        self.icl = None
        if args.icl_filter_model:
            from synthefy_nori_b200.training.icl_filter import ICLFilter
            from synthefy_nori_b200.utils.loading import load_model

            path = args.icl_filter_model
            if not os.path.exists(path):
                from synthefy_nori_b200.hf import download_checkpoint

                path = download_checkpoint(path)
            self.icl = ICLFilter(load_model(path), device, args.icl_filter_reg_min_r2, args.icl_filter_max_rounds)
        elif args.learnability_filter or args.icl_scaling_filter:
            from synthefy_nori_b200.training.icl_filter import TreeLearnabilityFilter

            self.icl = TreeLearnabilityFilter(args.learnability_filter_reg_min_score, args.icl_filter_max_rounds,
                                              scaling=args.icl_scaling_filter,
                                              min_improvement=args.icl_scaling_min_improvement,
                                              learnability=args.learnability_filter)
        self.prefetch = None
        if args.prefetch_workers > 0:
            import functools

            from synthefy_nori_b200.training.prefetch import DataPrefetcher

            spec = (args.prior, args.batch_size, self.shape_cfg, self.family_probs, args.augment, rank, args.seed)
            self.prefetch = DataPrefetcher(functools.partial(_host_batch, spec), args.prefetch_workers,
                                           base_seed=0)
        self.health = None
        if args.heartbeat_stale_s > 0 and world > 1:
            from synthefy_nori_b200.parallel.health import RankHealth

            self.health = RankHealth(dist.distributed_c10d._get_default_store(), rank, world,
                                     stale_s=args.heartbeat_stale_s)
        self.step = 0
        self.micro = 0

    # ------------------------------------------------------------------ checkpoint state
    def _flat_layout(self):
        tr = self.trainer
        if tr.peer is not None:
            return tr.peer.params, tr.peer.offsets
        return tr.flat.params, tr.flat.offsets

    def _per_param(self, full: torch.Tensor) -> dict:
        """Split a full flat vector into ``{parameter name: tensor}`` (layout-independent,
        so a checkpoint resumes under any world size or gradient path)."""
        names = {id(p): n for n, p in self.trainer.model.named_parameters()}
        params, offsets = self._flat_layout()
        return {names[id(p)]: full[o : o + p.numel()].view(p.shape).detach().cpu() for p, o in zip(params, offsets)}

    def _to_flat(self, per: dict, like: torch.Tensor) -> torch.Tensor:
        names = {id(p): n for n, p in self.trainer.model.named_parameters()}
        params, offsets = self._flat_layout()
        full = torch.zeros_like(like)
        for p, o in zip(params, offsets):
            full[o : o + p.numel()].copy_(per[names[id(p)]].reshape(-1).to(full))
        return full

    def state(self) -> dict:
        tr = self.trainer
        extra = {}
        if tr.peer is not None:
            m = self._per_param(tr.peer.full_from_owned(tr.peer.m))
            v = self._per_param(tr.peer.full_from_owned(tr.peer.v))
            ema = tr.peer.gather_ema()
            step = tr.peer.step_count
        elif tr.muon is not None:  # Muon: its own flat layout (same model + config on resume)
            m, v, ema, step = tr.opt.m.detach().cpu(), tr.opt.v.detach().cpu(), tr.opt.ema, tr.opt.step_count
            extra["muon_momentum"] = [b.detach().cpu() for _, _, b in tr.muon.groups]
        else:
            m, v = self._per_param(tr.opt.m), self._per_param(tr.opt.v)
            ema, step = tr.opt.ema, tr.opt.step_count
        sd = {k: t.detach().cpu() for k, t in tr.model.state_dict().items()}
        ema_sd = None
        if ema is not None:
            ema_sd = dict(sd)
            ema_sd.update(self._per_param(ema))
        health = tr.poll()
        return {
            "model_config": self.model_config,
            "model_state_dict": sd,
            "ema_state_dict": ema_sd,
            "optimizer_state": {"m": m, "v": v, "step": step, "layout": "per_parameter" if isinstance(m, dict)
                                else "muon_flat", **extra},
            "step": self.step,
            "training_config": dataclasses.asdict(self.tcfg) | {"argv": vars(self.args)},
            "rng_state": {"shape": self.shapes.state(), "torch": torch.get_rng_state()},
            "trainer_state": {"loss_ema": None if tr.loss_ema is None else float(tr.loss_ema),
                              "steps_done": tr.steps_done, "skipped_steps": health["skipped_steps"]},
        }

    def load(self, ckpt: dict) -> None:
        tr = self.trainer
        tr.model.load_state_dict(ckpt["model_state_dict"])  # also refreshes the bf16 layouts
        o = ckpt["optimizer_state"]
        ema_sd = ckpt.get("ema_state_dict")
        if tr.peer is not None:
            for k in ("m", "v"):
                getattr(tr.peer, k).copy_(tr.peer.owned_from_full(self._to_flat(o[k], tr.peer.data)))
            if tr.peer.ema is not None and ema_sd is not None:
                tr.peer.ema.copy_(tr.peer.owned_from_full(self._to_flat(ema_sd, tr.peer.data)))
            tr.peer.step_count = int(o["step"])
        elif tr.muon is not None:
            tr.opt.m.copy_(o["m"])
            tr.opt.v.copy_(o["v"])
            if tr.opt.ema is not None and ema_sd is not None:
                tr.opt.ema.copy_(self._to_flat(ema_sd, tr.flat.data))
            tr.opt.step_count = int(o["step"])
            for (_, _, b), src in zip(tr.muon.groups, o["muon_momentum"]):
                b.copy_(src)
        else:
            tr.opt.m.copy_(self._to_flat(o["m"], tr.opt.m))
            tr.opt.v.copy_(self._to_flat(o["v"], tr.opt.v))
            if tr.opt.ema is not None and ema_sd is not None:
                tr.opt.ema.copy_(self._to_flat(ema_sd, tr.flat.data))
            tr.opt.step_count = int(o["step"])
        self.step = int(ckpt["step"])
        ts = ckpt.get("trainer_state") or {}
        if ts.get("loss_ema") is not None:
            tr.loss_ema = torch.tensor(ts["loss_ema"], device=self.device)
        tr.steps_done = int(ts.get("steps_done", 0))
        tr.skipped_steps = int(ts.get("skipped_steps", 0))
        self.shapes.set_state(ckpt["rng_state"]["shape"])
        torch.set_rng_state(ckpt["rng_state"]["torch"])

    def _batch(self, rows, feats, ep, micro):
        a = self.args
        seed = (a.seed * 1_000_003 + self.step * 9973 + micro * 131 + self.rank) & 0x7FFFFFFF
        x, y = make_tables(a.prior, a.batch_size, rows, feats, ep, seed, self.device, self.family_probs, a.augment)
        if self.icl is not None:
            def regenerate(slots, rnd):
                xs, ys = make_tables(a.prior, len(slots), rows, feats, ep, (seed + 7777 * rnd) & 0x7FFFFFFF,
                                     self.device, self.family_probs, a.augment)
                return xs, ys

            x, y = self.icl.filter(x, y, ep, regenerate)
        return x, y

    def train_one(self):
        from synthefy_nori_b200.training.shapes import ShapeSampler

        a = self.args
        lr = wcd_lr(self.step, a.lr, a.warmup_steps, a.decay_start_step or int(0.8 * a.total_steps), a.total_steps,
                    a.min_lr_ratio)
        tr = self.trainer
        tr.set_lr(lr)
        if self.health is not None:
            self.health.beat(self.step)
            self.health.check(self.step)
        loss = None
        for micro in range(a.gradient_accumulation):
            if self.prefetch is not None:
                x, y, ep = next(self.prefetch)
                x, y = x.to(self.device, non_blocking=True), y.to(self.device, non_blocking=True)
            else:
                rows, feats, ratio = self.shapes.sample()
                ep = ShapeSampler.eval_pos(rows, ratio)
                x, y = self._batch(rows, feats, ep, micro)
            loss = tr.train_step(x, y, ep)
        self.step += 1
        return loss


def main(argv=None) -> int:
    args = parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device(args.device) if (args.device and world == 1) else torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        timeout = datetime.timedelta(seconds=int(os.environ.get("NCCL_TIMEOUT", "1800")))
        dist.init_process_group("nccl", timeout=timeout, device_id=device)
    run = Run(args, device, rank, world)
    if args.resume:
        path = args.resume
        if path == "latest":
            if not args.checkpoint_dir:
                raise SystemExit("--resume latest needs --checkpoint-dir")
            path = os.path.join(args.checkpoint_dir, "latest.pt")
        run.load(torch.load(path, map_location="cpu", weights_only=False))
        if rank == 0:
            print(f"resumed from {path} at step {run.step}", flush=True)
    stop = args.total_steps if args.run_steps is None else min(args.total_steps, run.step + args.run_steps)
    from synthefy_nori_b200.training.metrics import MetricsSink, PhaseTimer

    wandb_extra = {k: v for k, v in (("entity", args.wandb_entity), ("group", args.wandb_group),
                                       ("job_type", args.wandb_job_type),
                                       ("tags", args.wandb_tags.split(",") if args.wandb_tags else None))
                   if v is not None}
    sink = MetricsSink(args.metrics_file, rank, args.wandb_project, args.wandb_name,
                       config={k: v for k, v in vars(args).items() if isinstance(v, (int, float, str, bool))},
                       wandb_kwargs=wandb_extra)
    if rank == 0:
        for note in args.notices:
            print(f"note: {note}", flush=True)
    t0, last = time.time(), None
    try:
        while run.step < stop:
            diag = args.diagnostics_interval > 0 and (run.step + 1) % args.diagnostics_interval == 0
            if diag:
                with PhaseTimer() as timer:
                    last = run.train_one()
            else:
                last = run.train_one()
            if run.step % args.log_interval == 0 or run.step == stop or diag:
                run.trainer.raise_if_fatal()  # every rank: the decision is the same everywhere
                rec = {"loss": float(last.item()), "lr": wcd_lr(run.step - 1, args.lr, args.warmup_steps,
                                                                 args.decay_start_step or int(0.8 * args.total_steps),
                                                                 args.total_steps, args.min_lr_ratio),
                       "elapsed_s": round(time.time() - t0, 1)}
                rec.update(run.trainer.poll())
                if diag:
                    rec["phase_ms"] = timer.collect()  # max over ranks (collective)
                    rec["grad_norms"] = run.trainer.component_grad_norms()
                if run.icl is not None:
                    rec["icl_filter"] = dict(run.icl.stats)
                sink.log(rec, step=run.step)
            if args.checkpoint_dir and (run.step % args.save_interval == 0 or run.step == stop):
                st = run.state()  # collective in the sharded case: every rank takes part
                if rank == 0:
                    os.makedirs(args.checkpoint_dir, exist_ok=True)
                    _atomic_save(st, os.path.join(args.checkpoint_dir, "latest.pt"))
    finally:
        sink.close()
        if run.prefetch is not None:
            run.prefetch.close()
    if run.health is not None:
        run.health.leave()
    run.trainer.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
