"""Native (sm_100a) operator library.

``_C`` is the in-tree CUDA extension built by ``setup.py build_ext --inplace`` (or
``__graft_entry__.build()``).  Every op in this package calls into it on CUDA tensors
and raises if the extension is missing on a GPU box: there is no silent fallback.
"""

from __future__ import annotations

import torch  # noqa: F401  (loads libc10 / libtorch before the extension)

_C = None
_IMPORT_ERROR: str | None = None

try:  # pragma: no cover - depends on the build
    from synthefy_nori_b200 import _C  # type: ignore  # noqa: F811
except Exception as exc:  # noqa: BLE001
    _C = None
    _IMPORT_ERROR = f"{type(exc).__name__}: {exc}"


def native_available() -> bool:
    return _C is not None


def native_import_error() -> str | None:
    return _IMPORT_ERROR


def lib():
    if _C is None:
        raise RuntimeError(f"synthefy_nori_b200._C is not built or failed to load ({_IMPORT_ERROR})")
    return _C


from synthefy_nori_b200.ops.api import *  # noqa: E402,F401,F403
