"""Pytest configuration: the `gpu` marker and shared fixtures.

Tests marked gpu need a B200 (sm_100) and the in-tree libhs_ext.so; everything
else runs on the CPU (oracle vs golden vectors, host logic, ABI exports,
gloo multi-process paths).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden" / "golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the CUDA library")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="session")
def cuda_dev():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
