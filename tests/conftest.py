import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (sm_100a) and runs the CUDA kernels")


def _has_gpu() -> bool:
    try:
        from manifesto_b200 import device_count
        return device_count() > 0
    except Exception:
        return False


@pytest.fixture(scope="session")
def backend():
    """The CUDA backend on device 0 (fails loudly if the library is missing)."""
    from manifesto_b200 import CUDABackend
    if not _has_gpu():
        pytest.skip("no CUDA device visible")
    b = CUDABackend(0)
    yield b


@pytest.fixture(scope="session")
def ref():
    from oracle import ref as r
    r.lib()
    return r


@pytest.fixture(scope="session")
def golden():
    import json
    with open(ROOT / "tests" / "golden" / "reference_vectors.json") as f:
        return json.load(f)


def host_threads() -> int:
    return max(1, min(32, os.cpu_count() or 1))
