import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity tests of the CUDA path")


def has_gpu() -> bool:
    try:
        from dracomancer_llmengine_b200 import lib
        return lib().draco_b200_device_count() > 0
    except Exception:
        return False


@pytest.fixture(scope="session")
def port():
    from oracle.oracle import Port
    return Port()


@pytest.fixture(scope="session")
def ref():
    from oracle.oracle import Ref, ref_available
    if not ref_available():
        pytest.skip("oracle/_ref not built (reference sources absent)")
    return Ref()


@pytest.fixture(scope="session")
def dlib():
    from dracomancer_llmengine_b200 import lib
    L = lib()
    if L.draco_b200_device_count() <= 0:
        pytest.fail("GPU test run without a visible CUDA device")
    return L
