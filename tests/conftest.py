import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def rk_lib():
    from rokoko_b200 import lib
    return lib.load()


@pytest.fixture(scope="session")
def v1_blob():
    from rokoko_b200 import koko
    return koko.random_v1_blob(0)
