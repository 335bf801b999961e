import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
if str(ROOT / "tests") not in sys.path:
    sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and runs the CUDA kernels")


@pytest.fixture(scope="session")
def device():
    """The CUDA library on device 0; a GPU test fails (never skips) without one."""
    from tensorcrate_b200 import _native as N
    import ctypes as C

    n = C.c_int(0)
    N.call("tc_device_count", C.byref(n))
    assert n.value > 0, "no CUDA device visible"
    N.call("tc_set_device", 0)
    return N
