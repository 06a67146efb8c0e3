"""Test configuration: the `gpu` marker and shared helpers.

`-m "not gpu"` runs on any machine: the oracle against the reference's golden vectors, the
host-side logic, and that liblema_b200.so loads and exports its C ABI. `-m gpu` runs the
parity tests proper on a B200, through the C ABI, against the oracle and the golden vectors.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device (run with -m 'not gpu' on CPU)"
    return torch.device("cuda", 0)
