"""ORACLE TEST INFRASTRUCTURE -- ctypes access to oracle/_ref/libnnref.so.

libnnref.so is the reference's own NeuroNet.cl kernel source compiled for the
host CPU by oracle/build_ref.py.  `RefKernels.launch(name, global_size,
local_size, args)` executes one kernel over an NDRange exactly as the MQL5
host would enqueue it (`COpenCL::Execute`), with numpy float32 arrays for
buffer arguments and Python numbers for scalar arguments.

Only tests/, tests/golden/make_golden.py, __graft_entry__.smoke() and the CPU
baseline leg of bench.py use this module.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_ref", "libnnref.so")
# the same kernels with multiply-adds contracted into FMAs (OpenCL's default FP_CONTRACT ON)
LIB_FMA_PATH = os.path.join(HERE, "_ref", "libnnref_fma.so")


def host_has_fma() -> bool:
    """Whether this CPU executes the FMA instructions libnnref_fma.so is compiled with."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return " fma " in line + " "
    except OSError:
        pass
    return False


class RefKernels:
    def __init__(self, path: str = LIB_PATH):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (python oracle/build_ref.py)")
        lib = ctypes.CDLL(path)
        lib.nnref_kernel_name.restype = ctypes.c_char_p
        lib.nnref_kernel_argtypes.restype = ctypes.c_char_p
        lib.nnref_launch.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_size_t),
                                     ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_void_p)]
        lib.nnref_launch.restype = ctypes.c_int
        self.lib = lib
        self.sig = {}
        for i in range(lib.nnref_kernel_count()):
            self.sig[lib.nnref_kernel_name(i).decode()] = lib.nnref_kernel_argtypes(i).decode()

    @staticmethod
    def available(path: str = LIB_PATH) -> bool:
        return os.path.exists(path)

    def max_threads(self) -> int:
        return int(self.lib.nnref_max_threads())

    def launch(self, name: str, global_size, local_size, args) -> None:
        types = self.sig[name]
        if len(args) != len(types):
            raise ValueError(f"{name}: expected {len(types)} args, got {len(args)}")
        keep = []
        ptrs = (ctypes.c_void_p * len(args))()
        for i, (t, a) in enumerate(zip(types, args)):
            if t == "p":
                if not (isinstance(a, np.ndarray) and a.flags.c_contiguous and a.dtype == np.float32):
                    raise TypeError(f"{name} arg {i}: need a C-contiguous float32 array")
                ptrs[i] = a.ctypes.data
            elif t == "f":
                v = ctypes.c_float(float(a))
                keep.append(v)
                ptrs[i] = ctypes.addressof(v)
            elif t == "u":
                v = ctypes.c_uint(int(a))
                keep.append(v)
                ptrs[i] = ctypes.addressof(v)
            else:
                v = ctypes.c_int(int(a))
                keep.append(v)
                ptrs[i] = ctypes.addressof(v)
        g = list(global_size)
        dims = len(g)
        garr = (ctypes.c_size_t * dims)(*g)
        larr = None if local_size is None else (ctypes.c_size_t * dims)(*list(local_size))
        rc = self.lib.nnref_launch(name.encode(), dims, garr, larr, ptrs)
        if rc != 0:
            raise RuntimeError(f"nnref_launch({name}) failed: {rc}")
