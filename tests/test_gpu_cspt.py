"""CSP pipelines as device processes (-m gpu): one CTA per process, channels as counters in global memory.

The reference runs every process of a ``connect([...], [...])`` pipeline on its own thread
(src/python/pto_codegen.cpp:1759-2220).  The runtime runs such a body as one cooperative launch, one CTA per process,
each running its tasks through the tile-program interpreter in process order and its sends / receives on device
counters (bounded waits).  Each captured reference CSP case must give the reference's buffers and cycle count that
way, the same buffers as the dependency-wave form, and once more from the cached program; a pipeline whose
processes race on a tile runs as waves and still matches the oracle.
"""

import numpy as np
import pytest
from cpu_sim import CpuSim

from _cspt_cases import CASES, CSP_NAMES, racy_case
from golden_cases import case_index, expected_roots, materialize
from pto_wsp_b200.runtime import CudaExecutable

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", CSP_NAMES)
def test_reference_pipeline_as_device_processes(name, require_cuda):
    idx = case_index(CASES, name)
    case = CASES[idx]
    ex = CudaExecutable(case["plan"])
    outs = []
    for _ in range(2):  # the second run replays the cached program
        roots, arrays, axis, syms, sptr = materialize(case, idx)
        assert ex.run_with_symbols(arrays, axis, syms, sptr) == case["cycles"]
        assert ex.describe()["csp"] == "device_processes"
        assert ex.timing()["launches"] == 1
        for got, want in zip(roots, expected_roots(case, idx)):
            np.testing.assert_array_equal(got, want)  # copies and products: exact
        outs.append([r.copy() for r in roots])
    waves = CudaExecutable(case["plan"])
    waves.set_option("csp_device", 0)
    roots, arrays, axis, syms, sptr = materialize(case, idx)
    assert waves.run_with_symbols(arrays, axis, syms, sptr) == case["cycles"]
    assert waves.describe()["csp"] == "waves: csp_device option is 0"
    for a, b in zip(roots, outs[0]):
        np.testing.assert_array_equal(a, b)


def test_racy_pipeline_runs_as_waves_and_matches_the_oracle(require_cuda):
    case = racy_case()
    idx = case_index(CASES, "reftest:test_codegen_cspt_pipeline.py#0")
    roots, arrays, axis, syms, sptr = materialize(CASES[idx], idx)
    ref = [a.copy() for a in arrays]
    cycles = CpuSim(case["plan"]).run(ref)
    ex = CudaExecutable(case["plan"])
    assert ex.run_with_symbols(arrays, axis, syms, sptr) == cycles
    assert ex.describe()["csp"].startswith("waves: ")
    for got, want in zip(arrays, ref):
        np.testing.assert_array_equal(got, want)
