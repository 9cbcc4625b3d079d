import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
TESTS = Path(__file__).resolve().parent
if str(TESTS) not in sys.path:
    sys.path.insert(0, str(TESTS))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; runs the CUDA path")
    config.addinivalue_line("markers", "slow: large CPU oracle work")


@pytest.fixture(scope="session")
def fleet():
    return importlib.import_module("fleet-mi300x_b200")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(TESTS / "golden" / "golden_mla.npz"))


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail(f"GPU tests need sm_100 (B200); found compute capability {major}.x")
    return torch.device("cuda:0")
