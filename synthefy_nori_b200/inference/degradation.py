"""Warnings raised when inference quietly trades accuracy for feasibility, and a context
manager that turns them into errors (reference ``inference/degradation.py:45-101``)."""

from __future__ import annotations

import contextlib
import warnings


class DegradedPipelineWarning(UserWarning):
    """Base class: the prediction ran, but not exactly as configured."""


class SvdFallbackWarning(DegradedPipelineWarning):
    """A high-dimensional feature reduction fell back to a cheaper method."""


class ContextSubsampledWarning(DegradedPipelineWarning):
    """Context rows were dropped to fit the memory budget."""


class CacheQuantizedWarning(DegradedPipelineWarning):
    """The context cache was stored int8 although bf16 was requested."""


class MemoryEscalatedWarning(DegradedPipelineWarning):
    """An out-of-memory error moved the context cache to a lower rung (int8, host offload,
    streamed blocks) and the prediction was retried there."""


@contextlib.contextmanager
def strict_pipeline(*categories: type[Warning]):
    """Raise instead of warn for the given degradation categories (default: all)."""
    cats = categories or (DegradedPipelineWarning,)
    with warnings.catch_warnings():
        for c in cats:
            warnings.simplefilter("error", c)
        yield
