"""The oracle against the reference's golden values (CPU).

* Cycle counts the reference example drivers expect (their ``CycleCheck``s):
  e2e_rmsnorm 1072 (examples/e2e_rmsnorm/e2e_rmsnorm_example.py:32), softmax
  39848 (examples/softmax/softmax_example.py:32), bgemm 275968
  (examples/bgemm/bgemm_example.py:33), flashinfer_decode 4514
  (examples/flashinfer_decode/flashinfer_decode_example.py:35), indexer "pto"
  800 (examples/deepseek_lightning_indexer/deepseek_lightning_indexer_example.py:40).
  The survey reproduced these exactly on the reference CPU-sim.
* The captured fixtures replay bit-identically through the oracle.
* When the reference frontend is present, the reference's own scripts are re-run
  against the oracle by tests/golden/make_golden.py (see test_make_golden_*).
"""

import numpy as np
import pytest
from cpu_sim import CpuSim, Scheduler, stable_topk

from golden_cases import case_index, expected_roots, load_cases, materialize

CASES = load_cases()

EXPECTED_EXAMPLE_CYCLES = {
    "example:e2e_rmsnorm#0": 1072,
    "example:softmax#0": 39848,
    "example:bgemm#0": 275968,
    "example:flashinfer_decode#0": 4514,
    "example:deepseek_lightning_indexer#0": 800,
}


@pytest.mark.parametrize("name,cycles", sorted(EXPECTED_EXAMPLE_CYCLES.items()))
def test_example_cycles_pinned(name, cycles):
    i = case_index(CASES, name)
    assert CASES[i]["cycles"] == cycles


@pytest.mark.parametrize("idx", range(len(CASES)), ids=[c["name"] for c in CASES])
def test_oracle_replays_fixture(idx):
    case = CASES[idx]
    roots, arrays, axis, syms, sptr = materialize(case, idx)
    cycles = CpuSim(case["plan"]).run(arrays, axis, syms, sptr)
    assert cycles == case["cycles"]
    for got, want in zip(roots, expected_roots(case, idx)):
        np.testing.assert_array_equal(got, want)


def test_dispatch_window_semantics():
    # test_codegen_schedule_dispatch_window.py:11-60: rr(2) halves, window(1) serialises.
    s1 = Scheduler(1, 0)
    t1 = max(s1.issue(64, 0, 0) for _ in range(4))
    s2 = Scheduler(2, 0)
    t2 = 0
    for i in range(4):
        t2 = max(t2, s2.issue(64, i % 2, 0))
    s3 = Scheduler(2, 1)
    t3 = 0
    for i in range(4):
        t3 = max(t3, s3.issue(64, i % 2, 0))
    assert t2 * 2 == t1 and t3 == t1


def test_stable_topk_tie_rule():
    # examples/deepseek_lightning_indexer/golden.py:6-25: score desc, ties -> lower index.
    s = np.array([1.0, 3.0, 3.0, -0.0, 0.0, 2.0, 3.0], dtype=np.float32)
    assert stable_topk(s, 5).tolist() == [1, 2, 6, 5, 0]
    rng = np.random.default_rng(0)
    x = rng.integers(-4, 4, size=1000).astype(np.float32)
    order = np.lexsort((np.arange(x.size), -x.astype(np.float64)))
    assert stable_topk(x, 100).tolist() == order[:100].tolist()
