"""Locate and import the unmodified reference package (``baseline/_ref``).

The reference (``synthefy-nori``) is installed offline with ``pip install --no-deps
--target baseline/_ref``; its client package ``synthefy`` is copied next to it. Two of
its optional dependencies are not in this image: ``pyvinecopulib`` (vine-copula
multi-target, reference ``api.py:11``) and ``kditransform`` (one preprocessing worker).
Empty placeholder modules are registered for them so that ``import synthefy_nori``
succeeds; no code path used by the parity tests or the reference bench arm touches
either.  The reference's own files are never edited.
"""

from __future__ import annotations

import os
import sys
import types

_REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF_DIR = os.path.join(_REPO, "baseline", "_ref")


class _Unavailable:
    """Placeholder for a class of a missing optional dependency; using it raises."""

    def __init__(self, *a, **k):
        raise ImportError("optional dependency of the reference is not installed in this image")


def import_reference():
    """Return the reference ``synthefy_nori`` module, or ``None`` if not installed."""
    if not os.path.isdir(os.path.join(REF_DIR, "synthefy_nori")):
        return None
    if REF_DIR not in sys.path:
        sys.path.append(REF_DIR)
    for name in ("pyvinecopulib", "kditransform"):
        if name not in sys.modules:
            try:
                __import__(name)
            except ImportError:
                stub = types.ModuleType(name)
                if name == "kditransform":
                    stub.KDITransformer = _Unavailable
                sys.modules[name] = stub
    import synthefy_nori  # noqa: F401

    return synthefy_nori
