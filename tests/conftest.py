import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def cuda_lib():
    """Build (if stale) and load the CUDA library; GPU tests fail loudly if it cannot load."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    from skinny_mlx_b200 import build, _lib

    build.build()
    return _lib.lib()


@pytest.fixture
def dev():
    import torch

    return torch.device("cuda", 0)


def golden(name: str) -> Path:
    return GOLDEN / name


os.environ.setdefault("PYTHONHASHSEED", "0")
