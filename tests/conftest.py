"""Test configuration: markers, seeds and import paths.

Markers follow the reference's ``tests/conftest.py:58-62``; ``gpu`` tests need a
CUDA device and call the CUDA library through its C ABI; everything else runs
on the CPU (oracle vs golden fixtures, host logic, library symbol checks,
gloo multi-process tests).
"""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO / "oracle"))
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(Path(__file__).resolve().parent))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); calls libcbq through its C ABI")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(autouse=True)
def _seeds():
    np.random.seed(42)
    try:
        import torch
        torch.manual_seed(42)
    except ImportError:
        pass
