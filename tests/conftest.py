"""Test configuration: the `gpu` marker and shared fixtures.

`pytest -m "not gpu"` runs on a host without a GPU (oracle against the
reference's golden vectors, the C-ABI surface, host logic, gloo ranks);
`pytest -m gpu` runs the parity tests through the C-ABI on a B200.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def lib():
    import eshkol_transformer_b200 as etb
    return etb.load()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a host without CUDA")
    torch.cuda.init()
    return torch.device("cuda:0")
