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


@pytest.mark.parametrize("text,message", [("240,5x0,3\n-1,0,-1\n", "not an integer: '5x0'"),
                                          ("240,500\n-1\n", "one activation per layer"),
                                          ("240,0,3\n-1,0,-1\n", "layer sizes must be positive")])
def test_harness_rejects_a_malformed_network_file(binary, tmp_path, text, message):
    """The network file is checked before the library is initialised (no device work for a bad file)."""
    (tmp_path / "net.txt").write_text(text)
    r = subprocess.run([binary, "--dir", str(tmp_path), "--steps", "1"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1
    assert message in r.stderr
