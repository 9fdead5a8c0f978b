"""Shared pytest configuration.

``-m gpu`` tests need a CUDA device (a B200); everything else runs on a CPU-only
machine.  The repository root is put on sys.path so that the package, the
oracle and the golden-case definitions import without installation.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test is marked gpu and needs a CUDA device")
    return torch.device("cuda:0")
