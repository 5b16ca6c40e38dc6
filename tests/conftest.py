"""Shared pytest configuration: the ``gpu`` marker and small fixtures."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built extension")
    config.addinivalue_line("markers", "slow: long-running test")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def ref():
    """The unmodified reference (upstream rsl_rl) installed in baseline/_ref, used as the CPU oracle."""
    import baseline

    if not baseline.reference_available():
        pytest.skip("reference not installed in baseline/_ref")
    baseline.add_reference_to_path()
    import rsl_rl

    return rsl_rl
