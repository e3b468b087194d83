"""Pytest configuration: the ``gpu`` marker and shared fixtures.

``-m "not gpu"`` runs the CPU suite (oracle vs golden vectors, C-ABI symbol
checks, host logic, gloo multi-process tests). ``-m gpu`` runs the parity tests
of the CUDA kernels against the CPU oracle on a B200.
"""

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(42)
    yield
