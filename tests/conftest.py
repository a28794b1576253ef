"""Shared pytest configuration: the ``gpu`` marker and common fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs 2+ CUDA devices")


def pytest_collection_modifyitems(config, items):
    import torch

    have = torch.cuda.is_available()
    n = torch.cuda.device_count() if have else 0
    skip = pytest.mark.skip(reason="no CUDA device")
    skip2 = pytest.mark.skip(reason="needs 2+ CUDA devices")
    for it in items:
        if "gpu" in it.keywords and not have:
            it.add_marker(skip)
        if "multigpu" in it.keywords and n < 2:
            it.add_marker(skip2)


@pytest.fixture
def dev():
    return "cuda:0"
