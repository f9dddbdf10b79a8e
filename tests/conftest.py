import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
if str(ROOT / "tests") not in sys.path:
    sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built CUDA library")
    config.addinivalue_line("markers", "slow: long-running")


def _has_gpu() -> bool:
    try:
        import torch  # noqa: F401

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    # GPU tests are selected with -m gpu; without a device they fail loudly
    # instead of silently passing, except when explicitly deselected.
    pass


@pytest.fixture(scope="session")
def cuda_backend():
    from bitnetrs_b200 import CudaBackend

    # Models and caches created by tests hold references to the context; it is
    # released when the last of them goes away.
    yield CudaBackend(int(os.environ.get("BITNET_TEST_DEVICE", "0")))
