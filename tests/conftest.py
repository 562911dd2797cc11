import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libnn_b200.so")


@pytest.fixture(scope="session")
def ctx():
    """One library context for the whole GPU session."""
    from nn_in_trading_b200 import Context
    c = Context(0)
    yield c
    c.close()
