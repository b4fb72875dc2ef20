import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """The engine library and the CPU oracle, built in-tree if stale."""
    from sheep_b200 import build
    build.build()
    from tests import helpers
    helpers.build_oracle()
    yield
