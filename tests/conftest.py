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


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """How many compared elements needed each allowance of tests/parity.py in this run."""
    from tests.parity import DRIFT, STATS
    for label, st in DRIFT.items():
        terminalreporter.write_line(
            "drift {}: tensor {:.2e} (bound {:g}); element-wise p50 {:.1e} p99 {:.1e} max {:.1e}".format(
                label, st["tensor_rel"], st["bound"], st["elem_p50"], st["elem_p99"], st["elem_max"]))
    if STATS["checks"]:
        terminalreporter.write_line(
            "parity: {checks} tensors, {elements} elements compared; element-wise rel err > 1e-4: "
            "{elem_rtol_1e-4}; accepted by the TANH/SIGMOID floor: {deact_floor}; weights with a cancelled "
            "gradient that moved the other way: {cancelled_weights}; in-place changes checked: "
            "{delta_checks}".format(**STATS))
