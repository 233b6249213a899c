"""Named NoriCausal checkpoints (reference ``causal/registry.py``): explicit ``checkpoint=``,
then the model's environment variable, then the Hugging Face download.  The calibrated
edge-probability threshold is the published value for that checkpoint."""

from __future__ import annotations

import os
from pathlib import Path

NORI_CAUSAL_MODELS = {
    "noricausal-31m": {"env": "SYNTHEFY_NORICAUSAL_31M_CHECKPOINT", "repo_id": "Synthefy/Nori-Causal",
                       "filename": "noricausal_31m.pt", "threshold": 0.8656008543608323,
                       "arch": {"d": 352, "r": 176, "n_blocks": 6, "n_pooled_blocks": 15, "max_rows": 2048}},
}


def get_checkpoint_path_and_threshold(model: str = "noricausal-31m", checkpoint=None) -> tuple[Path, float | None]:
    entry = NORI_CAUSAL_MODELS.get(model)
    if entry is None and checkpoint is None:
        raise ValueError(f"unknown NoriCausal model {model!r}; choose one of {sorted(NORI_CAUSAL_MODELS)} or pass "
                         "checkpoint=")
    path = checkpoint or (os.environ.get(entry["env"]) if entry else None)
    if not path:
        from synthefy_nori_b200.hf import download_checkpoint

        path = download_checkpoint(entry["repo_id"], filename=entry["filename"])
    path = Path(path).expanduser()
    if not path.is_file():
        raise FileNotFoundError(f"NoriCausal checkpoint not found: {path}")
    return path, (entry["threshold"] if entry else None)
