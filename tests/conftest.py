"""pytest configuration: the `gpu` marker and shared fixtures.

`-m gpu` tests need a CUDA device (they run on a B200 box); everything else
runs on the CPU. GPU tests skip only when no CUDA device exists at all; on a
machine with a GPU a missing or failing native library is a test failure.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs through libgdn_b200.so")


def _have_cuda() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _have_cuda():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this machine")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
