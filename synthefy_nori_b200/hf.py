"""Checkpoint registry and Hugging Face Hub download (reference ``src/synthefy_nori/hf.py``).

``NORI_MODELS`` maps the released variant names to their hub repositories; the default
file inside each repository is ``nori.pt``. ``download_checkpoint`` returns a local path,
honouring ``SYNTHEFY_NORI_HF_REPO`` / ``SYNTHEFY_NORI_HF_FILENAME`` for the base model.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from pathlib import Path

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


@dataclass(frozen=True)
class HubCheckpoint:
    """A published checkpoint: hub repository + file, an optional environment variable
    that points at a local copy, and free-form metadata (calibrated thresholds,
    architecture notes)."""

    repo_id: str
    filename: str = DEFAULT_FILENAME
    env_var: str | None = None
    meta: dict = field(default_factory=dict)


def resolve_checkpoint(entry: HubCheckpoint | None, explicit=None) -> Path:
    """Local checkpoint file, from the first source that names one: the caller's
    ``explicit`` path, then ``entry.env_var``, then a hub download of ``entry``.  A named
    local path that does not exist is an error (never silently replaced by a download)."""
    for candidate in (explicit, os.environ.get(entry.env_var) if entry is not None and entry.env_var else None):
        if candidate:
            path = Path(candidate).expanduser()
            if not path.is_file():
                raise FileNotFoundError(f"checkpoint file does not exist: {path}")
            return path
    if entry is None:
        raise ValueError("no checkpoint source: pass a file path or a registered model name")
    return Path(download_checkpoint(entry.repo_id, filename=entry.filename))


LIMIX_REPO_ID = "stableai-org/LimiX-2M"
LIMIX_FILENAME = "LimiX-2M.ckpt"


def download_limix(cache_dir: str | None = None, token=None) -> str:
    """The LimiX-2M base checkpoint (reference ``hf.py:162``)."""
    return download_checkpoint(LIMIX_REPO_ID, filename=LIMIX_FILENAME, cache_dir=cache_dir, token=token)


def push_checkpoint(path: str, repo_id: str, filename: str = DEFAULT_FILENAME, token=None, *, private: bool = True,
                    create_repo: bool = True, commit_message: str | None = None) -> None:
    """Upload a checkpoint file to a hub repository (reference ``hf.py:180``)."""
    from huggingface_hub import HfApi

    api = HfApi(token=token)
    if create_repo:
        api.create_repo(repo_id, private=private, exist_ok=True, repo_type="model")
    api.upload_file(path_or_fileobj=path, path_in_repo=filename, repo_id=repo_id, commit_message=commit_message)


def download_cli(argv=None) -> int:
    """``synthefy-nori-b200-download``: fetch a checkpoint and print its local path."""
    import argparse

    ap = argparse.ArgumentParser(description="Download a Nori checkpoint")
    src = ap.add_mutually_exclusive_group()
    src.add_argument("--model", default="nori-6m", help="registry name (" + ", ".join(NORI_MODELS) + ")")
    src.add_argument("--repo-id", default=None)
    ap.add_argument("--filename", default=None)
    ap.add_argument("--cache-dir", default=None)
    ap.add_argument("--token", default=None)
    a = ap.parse_args(argv)
    print(download_checkpoint(a.repo_id or a.model, filename=a.filename, cache_dir=a.cache_dir, token=a.token))
    return 0


def upload_cli(argv=None) -> int:
    """``synthefy-nori-b200-upload``: push a checkpoint file to a hub repository."""
    import argparse

    ap = argparse.ArgumentParser(description="Upload a Nori checkpoint")
    ap.add_argument("checkpoint_path")
    ap.add_argument("--repo-id", required=True)
    ap.add_argument("--filename", default=None)
    ap.add_argument("--public", action="store_true")
    ap.add_argument("--token", default=None)
    ap.add_argument("--commit-message", default=None)
    ap.add_argument("--no-create-repo", action="store_true")
    a = ap.parse_args(argv)
    push_checkpoint(a.checkpoint_path, a.repo_id, a.filename or os.path.basename(a.checkpoint_path), a.token,
                    private=not a.public, create_repo=not a.no_create_repo, commit_message=a.commit_message)
    return 0
