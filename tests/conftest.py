import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA backend")


def gpu_available() -> bool:
    try:
        from metellus_b200.runtime import backend

        return backend.device_count() > 0
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda_device():
    """Fails (does not skip) when a GPU test runs without a usable device: the CUDA
    path must be the one that runs, never silently skipped."""
    from metellus_b200.runtime import backend

    n = backend.device_count()
    assert n > 0, "no CUDA device visible to libmetellus_cuda.so"
    backend.init()
    return backend.current_device()
