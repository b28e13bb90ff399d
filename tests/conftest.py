import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (sm_100a B200)")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA backend context on device 0 (GPU tests only)."""
    from tpt_infer_b200 import CudaBackend

    be = CudaBackend.new(0)
    assert be is not None, "no CUDA device"
    yield be
    be.close()
