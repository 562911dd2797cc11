"""Generate tests/golden/kernels.npz from the reference kernels.

Runs every case of tests/golden/cases.py through the reference's own
NeuroNet.cl kernels compiled for the CPU (oracle/_ref/libnnref.so, built by
oracle/build_ref.py from the reference checkout) and stores, per case, the
inputs and every array argument after the launch.  Run from the repository
root:

    python oracle/build_ref.py --reference <checkout> && python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys
import zlib

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.ref import RefKernels  # noqa: E402
from tests.golden.cases import all_cases, prepare_inputs  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kernels.npz")


def case_seed(name: str) -> int:
    return zlib.crc32(name.encode()) & 0x7FFFFFFF


def main() -> int:
    ref = RefKernels()
    store = {}
    for case in all_cases():
        args = prepare_inputs(case, case_seed(case.name))
        for i, a in enumerate(args):
            if isinstance(a, np.ndarray):
                store[f"{case.name}|in{i}"] = a.copy()
        ref.launch(case.kernel, case.gsize, case.lsize, args)
        for i, a in enumerate(args):
            if isinstance(a, np.ndarray):
                store[f"{case.name}|out{i}"] = a
    np.savez_compressed(OUT, **store)
    print(f"wrote {OUT}: {len(all_cases())} cases, {os.path.getsize(OUT) / 1024:.0f} KiB")
    return 0


if __name__ == "__main__":
    sys.exit(main())
