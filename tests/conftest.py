import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: multi-second CPU work")
    # Bring the in-tree native library up to date (no-op when current).
    from b200_gemm_b200 import build

    build.build_library()


def _has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu_handle():
    """One b200gemm handle on cuda:0 for the whole GPU session.

    Fails (does not skip) when the GPU or the native library is missing: a GPU
    test that silently skips would hide a missing CUDA path."""
    if not _has_gpu():
        pytest.fail("GPU test selected but torch.cuda.is_available() is False")
    from b200_gemm_b200 import Gemm

    h = Gemm(0)
    yield h
    h.close()


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle

    oracle.build()
    return oracle
