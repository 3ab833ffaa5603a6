from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
TESTS = Path(__file__).resolve().parent
for p in (str(ROOT), str(TESTS)):
    if p not in sys.path:
        sys.path.insert(0, p)

from __graft_entry__ import load_package  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def tm():
    return load_package()


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA; run with -m 'not gpu'")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail("these tests need an sm_100 (B200) device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def adapter(tm, cuda_device):
    tm.load_adapter()
    return tm
