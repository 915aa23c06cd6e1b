"""CSP pipelines (CSPT time semantics) on the host: the native walk against the oracle (no GPU).

The reference runs each process of a ``connect([...], [...])`` pipeline on a thread and returns the largest
process clock (src/python/pto_codegen.cpp:1611-1705, :1759-2220).  The captured reference cases (the CSP
example, whose script expects 114688 cycles, and tests/test_codegen_cspt_pipeline.py) are re-run here with other
channel depths and latencies: the native cycle model (dry run, no CUDA call) must give the oracle's number.
"""

import copy

import numpy as np
import pytest

from golden_cases import case_index, load_cases, materialize
from cpu_sim import CpuSim
from pto_wsp_b200.plan import fnv1a_64
from pto_wsp_b200.runtime import CudaExecutable, PtoWspCudaError

CASES = load_cases()
LAT = fnv1a_64("__pto_wsp_channel_latency_cycles")


def _with_depth(plan, depth):
    p = copy.deepcopy(plan)
    for c in p["body"]["channels"]:
        c["capacity"] = depth
    return p


@pytest.mark.parametrize("name", ["example:csp_pipeline#0", "reftest:test_codegen_cspt_pipeline.py#0"])
@pytest.mark.parametrize("depth", [0, 1, 2, 3])
@pytest.mark.parametrize("latency", [0, 7, 50])
def test_native_pipeline_clock_matches_oracle(name, depth, latency):
    idx = case_index(CASES, name)
    plan = _with_depth(CASES[idx]["plan"], depth)
    roots, arrays, axis, syms, sptr = materialize(CASES[idx], idx)
    syms = dict(syms)
    syms[LAT] = latency
    want = CpuSim(plan).run([a.copy() for a in arrays], axis, syms, sptr)
    ex = CudaExecutable(plan)
    ex.set_option("dry_run", 1)
    assert ex.run_with_symbols(arrays, axis, syms, sptr) == want


def test_pipeline_overlaps_and_latency_adds():
    idx = case_index(CASES, "example:csp_pipeline#0")
    assert CASES[idx]["cycles"] == 114688  # the value examples/csp_pipeline/csp_pipeline_example.py expects
    plan = CASES[idx]["plan"]
    roots, arrays, axis, syms, sptr = materialize(CASES[idx], idx)
    ex = CudaExecutable(plan)
    ex.set_option("dry_run", 1)
    c0 = ex.run_with_symbols(arrays, axis, {LAT: 0}, sptr)
    c50 = ex.run_with_symbols(arrays, axis, {LAT: 50}, sptr)
    assert c0 == 114688 and c50 > c0


def test_pipeline_data_through_the_oracle():
    idx = case_index(CASES, "reftest:test_codegen_cspt_pipeline.py#0")
    roots, arrays, axis, syms, sptr = materialize(CASES[idx], idx)
    x, tmp, y = arrays
    for depth in (0, 1, 4):
        y[...] = 0
        tmp[...] = 0
        CpuSim(_with_depth(CASES[idx]["plan"], depth)).run(arrays, axis, syms, sptr)
        np.testing.assert_array_equal(y, x * x)


def test_pipeline_deadlock_is_an_error():
    idx = case_index(CASES, "reftest:test_codegen_cspt_pipeline.py#0")
    plan = copy.deepcopy(CASES[idx]["plan"])
    plan["body"]["processes"][0]["produces"] = []  # the producer never closes its channel
    roots, arrays, axis, syms, sptr = materialize(CASES[idx], idx)
    with pytest.raises(RuntimeError, match="deadlock"):
        CpuSim(plan).run(arrays, axis, syms, sptr)
    ex = CudaExecutable(plan)
    ex.set_option("dry_run", 1)
    with pytest.raises(PtoWspCudaError, match="deadlock"):
        ex.run_with_symbols(arrays, axis, syms, sptr)
