"""pytest configuration: the ``gpu`` marker and the repository on sys.path.

``-m "not gpu"`` runs the oracle, host-logic and C-ABI tests on a CPU-only
machine; ``-m gpu`` runs the parity and failure-detection tests on a B200.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda_available():
    import torch

    return torch.cuda.is_available()
