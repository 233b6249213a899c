"""Prefetcher: ordered reproducible output, error forwarding, dead-worker detection."""

import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(__file__))

from synthefy_nori_b200.training.prefetch import DataPrefetcher  # noqa: E402


def test_order_and_reproducibility():
    import _prefetch_fns as f

    with DataPrefetcher(f.make_batch, num_workers=3, base_seed=10) as p:
        got = [next(p) for _ in range(6)]
    for i, g in enumerate(got):
        np.testing.assert_array_equal(g, f.make_batch(10 + i))


def test_error_forwarded():
    import _prefetch_fns as f

    p = DataPrefetcher(f.failing, num_workers=2)
    assert next(p) == 0 and next(p) == 1
    with pytest.raises(RuntimeError, match="bad table"):
        next(p)


def test_dead_worker_detected():
    import _prefetch_fns as f

    p = DataPrefetcher(f.dying, num_workers=1, timeout_s=30)
    with pytest.raises(RuntimeError, match="exited"):
        next(p)
