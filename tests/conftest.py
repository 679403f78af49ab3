"""Shared test configuration.

Markers: ``gpu`` -- needs a CUDA device (sm_100) and the built library.
CPU tests cover the oracle against the committed golden fixtures, host-side
argument checking of the C ABI, and multi-process (gloo) host logic.
"""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA sm_100 device")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test collected on a machine without CUDA")
    return torch.device("cuda", 0)
