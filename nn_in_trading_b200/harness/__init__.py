"""C++ hosts of the library: programs that drive the C ABI (include/nn_b200.h) the way a Linux
caller would, with no Python on the path.  `build()` compiles one with the system g++ against the
in-tree libnn_b200.so."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
INCLUDE = os.path.join(ROOT, "include")
LIBDIR = PKG  # libnn_b200.so is built in-tree next to the Python package


def build(name: str = "dense_online", out: str | None = None, extra_flags: tuple = ()) -> str:
    """Compile harness/<name>.cpp into `out` (default: next to the source) and return its path.
    The binary finds libnn_b200.so through its run path; raises with the compiler's output on failure."""
    src = os.path.join(HERE, name + ".cpp")
    out = out or os.path.join(HERE, name)
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", *extra_flags, "-I", INCLUDE, src, "-o", out,
           "-L", LIBDIR, "-l:libnn_b200.so", "-Wl,-rpath," + LIBDIR]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed for {src}:\n{r.stdout}\n{r.stderr}")
    return out
