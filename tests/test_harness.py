"""The C++ host (nn_in_trading_b200/harness/dense_online.cpp) compiles against include/nn_b200.h
and links against libnn_b200.so with no warning, uses only entry points the header declares, and
rejects bad arguments.  No compute calls: these run on machines without a GPU."""
import os
import shutil
import subprocess

import pytest

from nn_in_trading_b200 import api, harness
from tests.test_abi import declared_symbols

pytestmark = pytest.mark.skipif(shutil.which("g++") is None, reason="no g++ on this machine")


@pytest.fixture(scope="module")
def binary(tmp_path_factory):
    assert os.path.exists(api.LIB_PATH), "libnn_b200.so not built"
    return harness.build(out=str(tmp_path_factory.mktemp("harness") / "dense_online"), extra_flags=("-Werror",))


def test_harness_uses_only_declared_entry_points(binary):
    nm = subprocess.run(["nm", "-D", "--undefined-only", binary], capture_output=True, text=True, check=True)
    used = sorted({line.split()[-1] for line in nm.stdout.splitlines() if line.split()[-1].startswith("nn_")})
    assert used, "the harness calls no library entry point"
    assert set(used) <= set(declared_symbols()), f"not in include/nn_b200.h: {sorted(set(used) - set(declared_symbols()))}"
    for required in ["nn_init", "nn_kernel_create", "nn_set_arg_buffer", "nn_execute", "nn_buffer_read",
                     "nn_shutdown"]:
        assert required in used


@pytest.mark.parametrize("args", [[], ["--bogus"], ["--steps", "3"], ["--dir", "x"]])
def test_harness_rejects_bad_arguments(binary, args):
    r = subprocess.run([binary, *args], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1
    assert "dense_online:" in r.stderr and "usage" in r.stderr
