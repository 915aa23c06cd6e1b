"""The oracle against the reference's golden values (CPU).

* Cycle counts the reference example drivers expect (their ``CycleCheck``s):
  e2e_rmsnorm 1072 (examples/e2e_rmsnorm/e2e_rmsnorm_example.py:32), softmax
  39848 (examples/softmax/softmax_example.py:32), bgemm 275968
  (examples/bgemm/bgemm_example.py:33), flashinfer_decode 4514
  (examples/flashinfer_decode/flashinfer_decode_example.py:35), indexer "pto"
  800 (examples/deepseek_lightning_indexer/deepseek_lightning_indexer_example.py:40).
  The survey reproduced these exactly on the reference CPU-sim.
* The captured fixtures replay bit-identically through the oracle.
* The reference's own CPU-sim artifact (its generated workload_main.cpp and
  kernel_*.cpp, built against the clean-room pto-isa stand-in oracle/ptoisa and
  run through its own CodegenExecutable by tests/golden/make_golden.py) gave the
  same cycle count on every fixture; its output buffers equal the oracle's --
  bit for bit where no exp/rsqrt is involved, else within 1e-5 relative.
* When the reference frontend is present, the reference's own scripts are re-run
  against the oracle by tests/golden/make_golden.py (see test_make_golden_*).
"""

import numpy as np
import pytest
from cpu_sim import CpuSim, Scheduler, fma_f32, stable_topk

from golden_cases import artifact_roots, case_index, expected_roots, load_cases, materialize

CASES = load_cases()

EXPECTED_EXAMPLE_CYCLES = {
    "example:e2e_rmsnorm#0": 1072,
    "example:softmax#0": 39848,
    "example:bgemm#0": 275968,
    "example:flashinfer_decode#0": 4514,
    "example:deepseek_lightning_indexer#0": 800,
    "example:attention#0": 1680,  # examples/attention/attention_example.py:34
    "example:llama#0": 4752,  # examples/llama/llama_example.py:35
    "example:deepseek_v3#0": 1408,  # examples/deepseek_v3/deepseek_v3_example.py:35
    "example:validated_matmul#0": 4864,  # examples/validated_matmul/validated_matmul_example.py:33
    "example:tensor_data#0": 8192,  # examples/tensor_data/tensor_data_example.py:37
    "example:tensor_data#1": 6144,  # examples/tensor_data/tensor_data_example.py:45
    "example:csp_pipeline#0": 114688,  # examples/csp_pipeline/csp_pipeline_example.py:32
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


@pytest.mark.parametrize("idx", range(len(CASES)), ids=[c["name"] for c in CASES])
def test_oracle_matches_the_reference_cpu_sim_artifact(idx):
    case = CASES[idx]
    art = artifact_roots(case, idx)
    assert art is not None, "fixture without the artifact's outputs: regenerate with tests/golden/make_golden.py"
    roots, arrays, axis, syms, sptr = materialize(case, idx)
    CpuSim(case["plan"]).run(arrays, axis, syms, sptr)
    for got, want in zip(roots, art):
        if np.issubdtype(want.dtype, np.floating):
            w = want.astype(np.float64)
            floor = 1e-5 * float(np.sqrt(np.mean(np.nan_to_num(w) ** 2))) if w.size else 0.0
            np.testing.assert_allclose(got.astype(np.float64), w, rtol=1e-5, atol=floor)
        else:
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


def test_fma_f32_rounds_once():
    # f32 TMATMUL steps are fused multiply-adds: compare with exact rational arithmetic rounded to nearest even
    from fractions import Fraction

    def exact(a, b, c):
        x = Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c))
        f = np.float32(float(x))
        cands = [f, np.nextafter(f, np.float32(np.inf)), np.nextafter(f, np.float32(-np.inf))]
        return min(cands, key=lambda y: (abs(Fraction(float(y)) - x), int(np.array(y).view(np.int32)) & 1))

    rng = np.random.default_rng(1)
    n = 3000
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    c = (rng.standard_normal(n) * np.exp2(rng.integers(-30, 30, n))).astype(np.float32)
    c[:1000] = -(a[:1000] * b[:1000])  # results that are the product's rounding error
    got = fma_f32(a, b, c)
    assert all(got[i] == exact(a[i], b[i], c[i]) for i in range(n))
    # double rounding through f64 would land on the midpoint 1 + 2^-23 + 2^-24 and round to even (1 + 2^-22)
    a1, b1, c1 = np.float32(2**-12 * (1 + 2**-23)), np.float32(2**-12 * (1 - 2**-23)), np.float32(1 + 2**-23)
    assert fma_f32(np.array([a1]), np.array([b1]), np.array([c1]))[0] == c1
