"""Tiered pretraining curriculum.

Tier 1 trains from scratch on small tables; every later tier starts from the previous
tier's final checkpoint with the model weights only (a fresh optimizer and learning-rate
schedule) and widens the table shapes: larger tables (2, 3), a long-context specialist
(4: up to 56k rows, few features, one table per GPU with gradient accumulation) and
the both-large corner (5: rows and features large together under a 7M-element budget).
The numbers are the reference's published launch settings (``scripts/train.sh``,
``scripts/continue_training.sh``), kept as one table so a run can be reproduced.

``tier_args(t)`` gives the CLI arguments of a tier; ``python -m
synthefy_nori_b200.training.curriculum --run-root DIR [--start-tier 2 --end-tier 5]``
runs the tiers in order (each under ``torchrun`` when ``--nproc-per-node`` > 1).
"""

from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys

TIERS = {
    1: dict(total_steps=250_000, lr=2e-4, warmup=4000, decay_start=60_000, batch=24, accum=1, budget=250_000,
            min_samples=256, max_samples=2048, min_features=2, max_features=250, bias_s=1.5, bias_f=1.3),
    2: dict(total_steps=30_000, lr=1e-4, warmup=2000, decay_start=20_000, batch=8, accum=3, budget=500_000,
            min_samples=256, max_samples=4096, min_features=16, max_features=384, bias_s=2.2, bias_f=1.55),
    3: dict(total_steps=30_000, lr=5e-5, warmup=1000, decay_start=10_000, batch=4, accum=6, budget=800_000,
            min_samples=512, max_samples=8144, min_features=32, max_features=768, bias_s=2.5, bias_f=1.75),
    4: dict(total_steps=10_000, lr=5e-5, warmup=300, decay_start=4000, batch=1, accum=16, budget=1_600_000,
            min_samples=1024, max_samples=56_000, min_features=4, max_features=96, bias_s=2.8, bias_f=1.3),
    5: dict(total_steps=8000, lr=5e-5, warmup=250, decay_start=3000, batch=1, accum=16, budget=7_000_000,
            min_samples=1024, max_samples=33_000, min_features=16, max_features=1280, bias_s=2.0, bias_f=2.0),
}

# shared by every tier: the recipe (prior mixture, loss, optimizer, architecture)
SHARED = ["--model", "nori-6m", "--optimizer", "muon", "--muon-include-nd", "--ema-decay", "0.999",
          "--loss", "pinball", "--pinball-monotonicity-weight", "0.05", "--prior", "mixture",
          "--scm-prior-prob", "0.34", "--tree-prior-prob", "0.08", "--gp-prior-prob", "0.12",
          "--quadratic-surface-prob", "0.06", "--sparse-nonlinear-prob", "0.08", "--lookup-prior-prob", "0.04",
          "--cat-dominant-prob", "0.08", "--binary-prior-prob", "0.04", "--temporal-prior-prob", "0.10",
          "--clean-lowdim-prob", "0.06", "--augment"]


def tier_args(t: int, overrides: dict | None = None) -> list[str]:
    c = dict(TIERS[t])
    c.update(overrides or {})
    return SHARED + [
        "--total-steps", str(c["total_steps"]), "--lr", str(c["lr"]), "--warmup-steps", str(c["warmup"]),
        "--decay-start-step", str(c["decay_start"]), "--batch-size", str(c["batch"]),
        "--gradient-accumulation", str(c["accum"]), "--max-budget", str(c["budget"]),
        "--min-rows", str(c["min_samples"]), "--max-rows", str(c["max_samples"]),
        "--min-features", str(c["min_features"]), "--max-features", str(c["max_features"]),
        "--dim-bias-samples", str(c["bias_s"]), "--dim-bias-features", str(c["bias_f"]),
    ]


def final_checkpoint(tier_dir: str) -> str | None:
    path = os.path.join(tier_dir, "latest.pt")
    if os.path.isfile(path):
        return path
    found = sorted(glob.glob(os.path.join(tier_dir, "checkpoint_step_*.pt")), key=os.path.getmtime)
    return found[-1] if found else None


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="run the pretraining curriculum tier by tier")
    ap.add_argument("--run-root", required=True)
    ap.add_argument("--start-tier", type=int, default=1)
    ap.add_argument("--end-tier", type=int, default=5)
    ap.add_argument("--nproc-per-node", type=int, default=1)
    ap.add_argument("--steps-scale", type=float, default=1.0, help="multiply every tier's step counts (probes)")
    ap.add_argument("--dry-run", action="store_true")
    a = ap.parse_args(argv)
    for t in range(a.start_tier, a.end_tier + 1):
        out = os.path.join(a.run_root, f"tier{t}")
        ov = {}
        if a.steps_scale != 1.0:
            for k in ("total_steps", "warmup", "decay_start"):
                ov[k] = max(1, int(TIERS[t][k] * a.steps_scale))
        args = tier_args(t, ov) + ["--checkpoint-dir", out]
        if t > 1:
            seed = final_checkpoint(os.path.join(a.run_root, f"tier{t - 1}"))
            if seed is None and not a.dry_run:
                raise SystemExit(f"tier {t} needs a tier {t - 1} checkpoint under {a.run_root}")
            args += ["--init-from", seed or "<tier-checkpoint>"]
        if a.nproc_per_node > 1:
            cmd = [sys.executable, "-m", "torch.distributed.run", "--standalone", "--local-addr", "127.0.0.1",
                   "--nproc-per-node", str(a.nproc_per_node), "-m", "synthefy_nori_b200.training.cli"] + args
        else:
            cmd = [sys.executable, "-m", "synthefy_nori_b200.training.cli"] + args
        print(" ".join(cmd), flush=True)
        if not a.dry_run:
            subprocess.run(cmd, check=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
