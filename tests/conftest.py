import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN


@pytest.fixture(scope="session")
def built_library():
    """Builds libaspire_b200.so if stale and loads it (works without a GPU)."""
    from aspire_b200 import build
    from aspire_b200 import _capi

    if build.is_stale() and os.environ.get("ASPIRE_B200_NO_BUILD") != "1":
        build.build()
    return _capi.load_library()


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    return torch.device("cuda:0")
