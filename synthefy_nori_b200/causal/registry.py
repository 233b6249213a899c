"""Published NoriCausal checkpoints.

Each entry is a ``hf.HubCheckpoint``; the calibrated edge-probability threshold of a
checkpoint (a published constant) and its architecture travel in the entry's metadata.
Resolution order (shared with the regressor's checkpoints, ``hf.resolve_checkpoint``):
an explicit file, the entry's environment variable, a hub download.
"""

from __future__ import annotations

from pathlib import Path

from synthefy_nori_b200.hf import HubCheckpoint, resolve_checkpoint

NORI_CAUSAL_MODELS: dict[str, HubCheckpoint] = {
    "noricausal-31m": HubCheckpoint(
        repo_id="Synthefy/Nori-Causal", filename="noricausal_31m.pt", env_var="SYNTHEFY_NORICAUSAL_31M_CHECKPOINT",
        meta={"threshold": 0.8656008543608323,
              "arch": {"d": 352, "r": 176, "n_blocks": 6, "n_pooled_blocks": 15, "max_rows": 2048}}),
}


def resolve_causal_checkpoint(model: str = "noricausal-31m", checkpoint=None) -> tuple[Path, float | None]:
    """(checkpoint file, calibrated threshold or None for an unregistered file)."""
    entry = NORI_CAUSAL_MODELS.get(model)
    if entry is None and checkpoint is None:
        known = ", ".join(sorted(NORI_CAUSAL_MODELS))
        raise ValueError(f"{model!r} is not a registered NoriCausal model (registered: {known}); "
                         "give checkpoint= a file path to use another one")
    path = resolve_checkpoint(entry, checkpoint)
    return path, (entry.meta.get("threshold") if entry is not None else None)
