import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) device")


@pytest.fixture(scope="session")
def built():
    """Builds (if stale) the product library and the oracle; returns their paths."""
    from fronk_b200 import build as fbuild
    from oracle import build as obuild
    lib = fbuild.build()
    res = obuild.build()
    res["product"] = lib
    return res


@pytest.fixture(scope="session")
def oracle(built):
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def gpu(built):
    import fronk_b200 as fb
    if not fb.cuda_available():
        pytest.fail("no sm_100 device: the CUDA path must run in -m gpu tests")
    return fb
