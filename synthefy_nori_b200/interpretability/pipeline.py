"""Command line for ``NoriInterpreter``: rank, prune and distill one table, write a JSON
report (ranking, sweep, scores and the glass-box model's shape functions).

    python -m synthefy_nori_b200.interpretability.pipeline --demo diabetes
    python -m synthefy_nori_b200.interpretability.pipeline --csv data.csv --target price
    python -m synthefy_nori_b200.interpretability.pipeline --npz data.npz   # X, y [, feature_names]

Parity target: reference ``interpretability/glassbox/pipeline.py`` (demo tables from
scikit-learn's bundled datasets, CSV with a target column, npz arrays; one JSON per run
under ``--out-dir``).  Non-numeric CSV columns are ordinal-encoded.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

from synthefy_nori_b200.interpretability.interpreter import NoriInterpreter


def load_table(a):
    if a.demo:
        from sklearn import datasets

        loader = {"diabetes": datasets.load_diabetes, "breast_cancer": datasets.load_breast_cancer}[a.demo]
        b = loader()
        return np.asarray(b.data, np.float32), np.asarray(b.target), list(b.feature_names), a.demo
    if a.csv:
        import pandas as pd

        df = pd.read_csv(a.csv)
        if a.target not in df.columns:
            raise SystemExit(f"--target {a.target!r} is not a column of {a.csv}")
        y = df.pop(a.target).to_numpy()
        for c in df.columns:
            if not pd.api.types.is_numeric_dtype(df[c]):
                df[c] = pd.Categorical(df[c]).codes.astype(np.float32)
                df.loc[df[c] < 0, c] = np.nan
        return df.to_numpy(np.float32), y, [str(c) for c in df.columns], os.path.splitext(os.path.basename(a.csv))[0]
    z = np.load(a.npz, allow_pickle=False)
    if "X" in z:
        X, y = z["X"], z["y"]
    else:  # pre-split arrays are joined; the interpreter makes its own split
        X, y = np.concatenate([z["Xtr"], z["Xte"]]), np.concatenate([z["ytr"], z["yte"]])
    names = [str(n) for n in z["feature_names"]] if "feature_names" in z else None
    return np.asarray(X, np.float32), y, names, os.path.splitext(os.path.basename(a.npz))[0]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="feature importance, pruning and glass-box distillation")
    src = ap.add_mutually_exclusive_group(required=True)
    src.add_argument("--demo", choices=["diabetes", "breast_cancer"])
    src.add_argument("--csv")
    src.add_argument("--npz")
    ap.add_argument("--target")
    ap.add_argument("--tag")
    ap.add_argument("--out-dir", default="explainability_out")
    ap.add_argument("--model", default="nori-6m")
    ap.add_argument("--weights", default=None, help="'random' for an offline run without a checkpoint")
    ap.add_argument("--device", default=None)
    ap.add_argument("--method", choices=["permutation", "shap"], default="permutation")
    ap.add_argument("--retain", type=float, default=0.95)
    ap.add_argument("--reduce-threshold", type=int, default=16)
    ap.add_argument("--test-size", type=float, default=0.3)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    if a.csv and not a.target:
        ap.error("--csv needs --target")
    X, y, names, tag = load_table(a)
    kw = {k: v for k, v in (("weights", a.weights), ("device", a.device)) if v is not None}
    interp = NoriInterpreter(a.model, method=a.method, retain=a.retain, reduce_threshold=a.reduce_threshold,
                             test_size=a.test_size, random_state=a.seed, regressor_kwargs=kw, verbose=True)
    interp.fit(X, y, feature_names=names)
    os.makedirs(a.out_dir, exist_ok=True)
    out = os.path.join(a.out_dir, f"{a.tag or tag}.json")
    rep = dict(interp.summary(), ranking=interp.importance_ranking_, selected=interp.selected_features_,
               glassbox=interp.ebm_model_)
    with open(out, "w") as f:
        json.dump(rep, f, indent=1, default=float)
    print(json.dumps({k: rep[k] for k in ("task", "metric", "n_selected", "nori_full", "ebm_selected")}, default=float))
    return 0


if __name__ == "__main__":
    sys.exit(main())
