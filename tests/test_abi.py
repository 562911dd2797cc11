"""The C-ABI shared library loads and exports every entry point include/nn_b200.h declares.

No compute calls: these run on machines without a GPU.
"""
import ctypes
import os
import re

import pytest

from nn_in_trading_b200 import api

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nn_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"NN_API\s+[\w\s\*]*?\b(nn_\w+)\s*\(", text)))


def test_header_declares_the_reference_boundary():
    names = declared_symbols()
    # COpenCLMy / COpenCL roles (NeuroNet_Declarations.mqh:359-513)
    for required in ["nn_init", "nn_shutdown", "nn_last_error", "nn_buffer_create", "nn_buffer_free",
                     "nn_buffer_write", "nn_buffer_read", "nn_kernel_create", "nn_set_arg_buffer",
                     "nn_set_arg_int", "nn_set_arg_float", "nn_execute", "nn_finish", "nn_max_local_size"]:
        assert required in names


def test_library_loads_and_exports_every_declared_symbol():
    assert os.path.exists(api.LIB_PATH), "libnn_b200.so not built"
    lib = ctypes.CDLL(api.LIB_PATH)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_covers_every_declared_symbol():
    lib = api.load_library()
    for n in declared_symbols():
        fn = getattr(lib, n)
        assert fn.restype is not None or n in ("nn_stream",), n


def test_every_reference_kernel_name_has_a_signature():
    from oracle.build_ref import KERNELS
    missing = [k for k in KERNELS if k not in api.SIGNATURES]
    assert not missing


def test_missing_library_fails_loudly(tmp_path):
    api_mod = api
    saved = api_mod._LIB
    try:
        api_mod._LIB = None
        with pytest.raises(api.NNError):
            api_mod.load_library(str(tmp_path / "nope.so"))
    finally:
        api_mod._LIB = saved
