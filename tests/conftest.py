"""pytest configuration: the ``gpu`` marker and shared fixtures."""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def golden_small():
    from golden_lib import load_small
    return load_small()


@pytest.fixture(scope="session")
def golden_pins():
    from golden_lib import load_pins
    return load_pins()
