import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "cuda-kernel_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: multi-process or large-shape test")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if gpu_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session", autouse=True)
def _native_builds():
    """Build the oracle (and the product libraries if absent) once per session."""
    import oracle
    if not oracle.LIB_PATH.exists():
        oracle.build(reference=True)
    from swiglu_b200 import _lib
    if not _lib.LIB_PATH.exists() or not _lib.CUBLAS_LIB_PATH.exists():
        if os.environ.get("SWB_NO_BUILD"):
            pytest.exit("native libraries missing and SWB_NO_BUILD is set")
        _lib.build()
    yield
