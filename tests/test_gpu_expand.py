"""Ragged axes and sparse selections expanded on the device (-m gpu).

A workload that is one loop over a ragged axis (reference `ParallelFor` over `Ragged`,
src/python/pto_codegen.cpp:2305-2416) or over a sparse selection (`Select`, :2417-2457) with one task as its body
is walked on the host once; a later run with other lengths or another selection keeps the cached task table and
rebuilds the loop's task records on the device from the new count or indices -- no host walk, no record upload
(`ptowsp_timing.walks == 0`, `expansions == 1`).  The makespan, which the entry ABI returns synchronously, is
recomputed on the host from the new task count with the same Scheduler::issue model (it needs the count only).
Every run matches the oracle bit for bit, makespan included.  The workloads are the reference's own
`tests/test_codegen_ragged_axis.py` and `tests/test_codegen_select_sparse.py` plans, captured as fixtures.
"""

import numpy as np
import pytest
from cpu_sim import CpuSim

from golden_cases import case_index, load_cases, materialize
from pto_wsp_b200.runtime import CudaExecutable

pytestmark = pytest.mark.gpu
CASES = load_cases()


def run_both(ex, plan, arrays, axis, syms, sptr):
    got = [a.copy() for a in arrays]
    want = [a.copy() for a in arrays]
    cycles = ex.run_with_symbols(got, axis, syms, {k: v for k, v in sptr.items()})
    want_cycles = CpuSim(plan).run(want, axis, syms, sptr)
    assert cycles == want_cycles
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g, w)
    t = ex.timing()
    return t["walks"], t["expansions"], t["tasks"]


def test_ragged_lengths_change_without_a_host_walk(require_cuda):
    idx = case_index(CASES, "reftest:test_codegen_ragged_axis.py#0")
    case = CASES[idx]
    roots, arrays, axis, syms, sptr = materialize(case, idx)
    (lens_id,) = sptr
    (outer_id,) = syms
    ex = CudaExecutable(case["plan"])
    assert run_both(ex, case["plan"], arrays, axis, syms, sptr) == (1, 0, 2)  # first run: the host walk
    for lengths, total in (([1, 2], 3), ([2, 1], 3), ([0, 1], 1), ([1, 2], 3)):
        s = {lens_id: np.asarray(lengths, np.int32)}
        walks, expansions, tasks = run_both(ex, case["plan"], arrays, axis, syms, s)
        assert walks == 0 and tasks == total
        # a new total rebuilds the records on the device; the same total replays them as they are
        assert expansions == (0 if lengths == [2, 1] else 1)


def test_sparse_selection_changes_without_a_host_walk(require_cuda):
    idx = case_index(CASES, "reftest:test_codegen_select_sparse.py#0")
    case = CASES[idx]
    roots, arrays, axis, syms, sptr = materialize(case, idx)
    (outer_id,) = syms
    body = case["plan"]["body"]
    indices_id, indptr_id = int(body["indices_sym"], 16), int(body["indptr_sym"], 16)
    ex = CudaExecutable(case["plan"])
    assert run_both(ex, case["plan"], arrays, axis, syms, sptr)[:2] == (1, 0)
    for outer, indptr, indices in ((1, [0, 1], [3]), (2, [0, 1, 4], [2, 0, 3, 1]), (1, [0, 2], [1, 3])):
        s = {indices_id: np.asarray(indices, np.int32), indptr_id: np.asarray(indptr, np.int32)}
        walks, expansions, tasks = run_both(ex, case["plan"], arrays, axis, {outer_id: outer}, s)
        assert (walks, expansions, tasks) == (0, 1, len(indices))
    # a repeated index while the kernel writes: the two tasks hit the same tile, so the host walk orders them
    s = {indices_id: np.asarray([2, 2], np.int32), indptr_id: np.asarray([0, 2], np.int32)}
    walks, expansions, _ = run_both(ex, case["plan"], arrays, axis, {outer_id: 1}, s)
    assert (walks, expansions) == (1, 0)
