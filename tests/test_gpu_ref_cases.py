"""Every captured reference case replayed on the GPU through the C ABI (-m gpu).

Cases come from the reference's own example drivers and codegen tests
(tests/golden/make_golden.py).  Each must give the oracle's buffers -- exactly
where the reference test demands atol=0, else within the example's tolerance
-- and the CPU-sim's exact cycle count.
"""

import numpy as np
import pytest

from golden_cases import expected_roots, load_cases, materialize
from pto_wsp_b200.runtime import CudaExecutable

CASES = load_cases()
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("idx", range(len(CASES)), ids=[c["name"] for c in CASES])
def test_reference_case_on_gpu(idx, require_cuda):
    case = CASES[idx]
    roots, arrays, axis, syms, sptr = materialize(case, idx)
    ex = CudaExecutable(case["plan"])
    cycles = ex.run_with_symbols(arrays, axis, syms, sptr)
    assert cycles == case["cycles"]
    for got, want in zip(roots, expected_roots(case, idx)):
        if np.issubdtype(want.dtype, np.floating) and (case["rtol"] or case["atol"]):
            np.testing.assert_allclose(got.astype(np.float64), want.astype(np.float64), rtol=case["rtol"],
                                       atol=case["atol"])
        else:
            np.testing.assert_array_equal(got, want)


def test_reference_case_twice_reuses_cached_task_table(require_cuda):
    idx = next(i for i, c in enumerate(CASES) if c["name"] == "example:e2e_rmsnorm#0")
    case = CASES[idx]
    ex = CudaExecutable(case["plan"])
    for _ in range(3):
        roots, arrays, axis, syms, sptr = materialize(case, idx)
        assert ex.run_with_symbols(arrays, axis, syms, sptr) == case["cycles"]
        for got, want in zip(roots, expected_roots(case, idx)):
            np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
