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


# ---- device processes: which pipelines the runtime runs as one CTA per process (dry run, no CUDA call) ----


def _dry_describe(plan, idx):
    roots, arrays, axis, syms, sptr = materialize(CASES[idx], idx)
    ex = CudaExecutable(plan)
    ex.set_option("dry_run", 1)
    cycles = ex.run_with_symbols(arrays, axis, syms, sptr)
    return cycles, ex.describe().get("csp"), ex


@pytest.mark.parametrize("name", ["example:csp_pipeline#0", "reftest:test_codegen_cspt_pipeline.py#0",
                                  "reftest:test_codegen_cspt_pipeline.py#2", "reftest:test_codegen_cspt_pipeline.py#3"])
def test_reference_pipelines_run_as_device_processes(name):
    # interpreter-runnable tasks, one sender and one receiver per channel, every cross-process hazard ordered by
    # the channels (vector clocks over the device's channel rules): one CTA per process, the walk's clock unchanged
    idx = case_index(CASES, name)
    cycles, mode, ex = _dry_describe(CASES[idx]["plan"], idx)
    assert mode == "device_processes" and cycles == CASES[idx]["cycles"]
    ex.set_option("csp_device", 0)
    assert ex.run_with_symbols(*materialize(CASES[idx], idx)[1:]) == CASES[idx]["cycles"]
    assert ex.describe()["csp"] == "waves: csp_device option is 0"


def test_racy_pipeline_runs_as_waves():
    # the producer runs ahead of a 4-deep channel and stores into the tile the consumer also stores after its first
    # receive: nothing orders those stores on the device, so the pipeline keeps the walk's order as waves
    from _cspt_cases import racy_case

    idx = case_index(CASES, "reftest:test_codegen_cspt_pipeline.py#0")
    cycles, mode, _ = _dry_describe(racy_case()["plan"], idx)
    assert mode == "waves: two processes write a tile in an order the channels do not fix"


def test_non_pipeline_body_has_no_csp_mode():
    idx = case_index(CASES, "reftest:test_codegen_cspt_pipeline.py#1")
    _, mode, _ = _dry_describe(CASES[idx]["plan"], idx)
    assert mode is None
