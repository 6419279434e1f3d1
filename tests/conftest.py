import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "pocket-workbench-android_b200")
for p in (ROOT, PKG_DIR, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200 / sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU oracle comparison")


@pytest.fixture(scope="session")
def oracle():
    import pko

    pko.lib()
    return pko


@pytest.fixture(scope="session")
def pk():
    """The product binding; GPU tests require the CUDA library to load."""
    import pocketinfer

    return pocketinfer
