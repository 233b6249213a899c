"""Checkpoint registry and Hugging Face Hub download (reference ``src/synthefy_nori/hf.py``).

``NORI_MODELS`` maps the released variant names to their hub repositories; the default
file inside each repository is ``nori.pt``. ``download_checkpoint`` returns a local path,
honouring ``SYNTHEFY_NORI_HF_REPO`` / ``SYNTHEFY_NORI_HF_FILENAME`` for the base model.
"""

from __future__ import annotations

import os

DEFAULT_FILENAME = "nori.pt"
NORI_MODELS = {
    "nori-6m": os.environ.get("SYNTHEFY_NORI_HF_REPO", "Synthefy/Nori"),
    "nori-1-5": "Synthefy/Nori-1-5",
    "nori-30m": "Synthefy/Nori-30M",
    "nori-100m": "Synthefy/Nori-100M",
}


def repo_for(model: str) -> str:
    """Registry lookup; an unknown name is treated as a raw ``org/repo`` id."""
    return NORI_MODELS.get(model, model)


def download_checkpoint(model: str = "nori-6m", filename: str | None = None, cache_dir: str | None = None,
                        token=None) -> str:
    """Local path of the checkpoint for ``model`` (downloaded and cached on first use)."""
    if os.path.isfile(model):
        return model
    fn = filename or (os.environ.get("SYNTHEFY_NORI_HF_FILENAME") if model == "nori-6m" else None) or DEFAULT_FILENAME
    try:
        from huggingface_hub import hf_hub_download
    except ImportError as exc:  # pragma: no cover
        raise RuntimeError("huggingface_hub is required to download checkpoints; pass model_path=") from exc
    try:
        return hf_hub_download(repo_id=repo_for(model), filename=fn, cache_dir=cache_dir, token=token)
    except Exception as exc:  # noqa: BLE001
        raise RuntimeError(
            f"could not fetch {repo_for(model)}/{fn} ({type(exc).__name__}: {exc}); pass model_path= to a local "
            "checkpoint or weights='random' for a random-init model"
        ) from exc


def push_checkpoint(path: str, repo_id: str, filename: str = DEFAULT_FILENAME, token=None) -> None:
    """Upload a checkpoint file to a hub repository (reference ``hf.py:push_checkpoint``)."""
    from huggingface_hub import HfApi

    HfApi(token=token).upload_file(path_or_fileobj=path, path_in_repo=filename, repo_id=repo_id)
