import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running test")


@pytest.fixture(scope="session")
def reference_pkg():
    """The unmodified reference package installed under ``baseline/_ref`` (skip if absent)."""
    from synthefy_nori_b200.utils.reference import import_reference

    mod = import_reference()
    if mod is None:
        pytest.skip("reference package not installed under baseline/_ref")
    return mod
