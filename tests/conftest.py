"""Shared test configuration.

Markers: ``gpu`` — needs a CUDA device (a B200: the library targets sm_100a).
CPU tests cover the oracle against the reference's golden vectors, the host
logic (argument checks, sharding plan, gloo all-gather) and the C ABI's
exported symbols; GPU tests are the parity tests proper.
"""

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected on a machine without CUDA")
    return torch.device("cuda:0")
