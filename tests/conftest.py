"""Test configuration: the ``gpu`` marker selects tests that need a B200."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "multirank: spawns several CPU (gloo) ranks")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def native():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from difflet_b200 import _native

    return _native.require()
