import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built libwamffn.so")


def pytest_sessionstart(session):
    torch.set_num_threads(max(1, min(8, os.cpu_count() or 1)))


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return torch.load(GOLDEN / name, weights_only=False)

    return load


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"sm_100 device required, found sm_{major}{minor}")
    from waminfer_b200 import _lib

    _lib.lib()  # loads libwamffn.so or raises: GPU tests never run without it
    return torch.device("cuda", 0)
