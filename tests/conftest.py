import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and libxgb.so")
    config.addinivalue_line("markers", "slow: long-running")


def golden(name: str):
    """Load a committed fixture (tests/golden/<name>.npz)."""
    return np.load(GOLDEN / f"{name}.npz")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is not available")
    major, _ = torch.cuda.get_device_capability()
    if major != 10:
        pytest.fail(f"xgen_b200 kernels target sm_100; found sm_{major}x")
    return torch.device("cuda", 0)
