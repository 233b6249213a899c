"""``python -m synthefy_nori_b200.evaluation.cli`` (reference ``evaluation/cli.py:16-123``)."""

from __future__ import annotations

import argparse
import sys


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Evaluate Nori checkpoints on regression benchmarks")
    ap.add_argument("--checkpoint", action="append", default=[], help="checkpoint path or label:path (repeatable)")
    ap.add_argument("--model", action="append", default=[], help="preset with random weights, e.g. nori-6m")
    ap.add_argument("--custom-reg-dir", action="append", default=[], help="dir of <name>_train.csv[/_test.csv]")
    ap.add_argument("--openml-list", default=None, help="pinned name,openml_dataset_id list (needs network)")
    ap.add_argument("--synthetic", action="store_true", help="add the offline synthetic suite")
    ap.add_argument("--output-dir", default="results/eval")
    ap.add_argument("--max-train-samples", type=int, default=50_000)
    ap.add_argument("--warmup", type=int, default=0)
    ap.add_argument("--no-cache", action="store_true")
    ap.add_argument("--device", default=None)
    a = ap.parse_args(argv)
    from synthefy_nori_b200.evaluation.datasets import DatasetRegistry
    from synthefy_nori_b200.evaluation.runner import EvalRunner, nori_model_fn

    reg = DatasetRegistry(max_train_samples=a.max_train_samples)
    for d in a.custom_reg_dir:
        reg.load_csv_dir(d)
    if a.openml_list:
        reg.load_openml(a.openml_list)
    if a.synthetic or not reg.datasets:
        reg.load_synthetic()
    models = {}
    for c in a.checkpoint:
        label, _, path = c.rpartition(":") if ":" in c else (c, "", c)
        models[label or path] = nori_model_fn(model_path=path, device=a.device)
    for m in a.model:
        models[m] = nori_model_fn(model=m, weights="random", device=a.device)
    if not models:
        ap.error("pass --checkpoint or --model")
    df = EvalRunner(models, reg.datasets, a.output_dir, warmup_runs=a.warmup, no_cache=a.no_cache).run()
    print(EvalRunner.summary(df).to_string())
    return 0


if __name__ == "__main__":
    sys.exit(main())
