"""Test configuration: the ``gpu`` marker and import paths.

``pytest -m "not gpu"`` runs on a CPU-only host (oracle vs golden fixtures,
host logic, the C-ABI library's exports and argument checks). ``pytest -m gpu``
needs a B200 and compares the CUDA kernels with the oracle through the C ABI.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
