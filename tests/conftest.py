import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built library")


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        return np.load(GOLDEN / name, allow_pickle=False)
    return load


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device; a GPU test without one fails instead of passing silently."""
    import torch
    if not torch.cuda.is_available():
        if os.environ.get("CAST_ALLOW_GPU_SKIP") == "1":
            pytest.skip("no CUDA device")
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda", 0)
