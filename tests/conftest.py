import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and runs the CUDA path")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Both native libraries, built once per session (no-op when up to date)."""
    from oracle import build as ob
    from pyxis_b200 import build as pb

    ob.build()
    pb.build()
    yield
