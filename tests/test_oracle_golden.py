"""The numpy oracle against the golden vectors made by the reference kernels.

tests/golden/kernels.npz holds, for every case of tests/golden/cases.py, the
outputs of the reference's own NeuroNet.cl kernels compiled for the CPU
(oracle/_ref, see tests/golden/make_golden.py).  This pins the restatement in
oracle/kernels.py before it is trusted as the checker of the CUDA library.
"""
import os

import numpy as np
import pytest

from oracle import kernels as K
from tests.golden.cases import all_cases, prepare_inputs
from tests.golden.make_golden import case_seed
from tests.parity import check_close

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kernels.npz")
CASES = all_cases()


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_oracle_matches_reference_kernels(case, golden):
    args = prepare_inputs(case, case_seed(case.name))
    before = [a.copy() if isinstance(a, np.ndarray) else None for a in args]
    for i, a in enumerate(args):
        if isinstance(a, np.ndarray):
            np.testing.assert_array_equal(a, golden[f"{case.name}|in{i}"])
    K.launch(case.kernel, case.gsize, case.lsize, args)
    for i, a in enumerate(args):
        if isinstance(a, np.ndarray):
            check_close(f"{case.name} arg{i}", a, golden[f"{case.name}|out{i}"], before[i])


def test_every_in_scope_kernel_has_golden_cases():
    covered = {c.kernel for c in CASES}
    restated = set(K.KERNELS) - K.LIBRARY_KERNELS
    missing = restated - covered
    assert not missing, f"restated kernels without golden cases: {sorted(missing)}"
