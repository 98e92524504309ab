import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) device")
    config.addinivalue_line("markers", "slow: long CPU test")


@pytest.fixture(scope="session")
def olib():
    import oracle
    return oracle.lib()


@pytest.fixture(scope="session")
def rlib():
    import oracle
    if not oracle.ref_available():
        pytest.skip("reference build (oracle/_ref) unavailable")
    return oracle.ref()
