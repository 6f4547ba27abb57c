import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope="session")
def cuda():
    """Skip unless a CUDA device is present; GPU tests are also marked ``gpu``."""
    if not cuda_available():
        pytest.skip("CUDA is required")
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    return torch.device("cuda", int(os.environ.get("FOCAL_TEST_DEVICE", "0")))
