"""The C port of the CPU-sim task bodies (oracle/cpu_kernels.c) against the numpy oracle (oracle/cpu_sim.py).

The port is the CPU baseline and the full-size checker of the GPU parity tests (every tile of configs 1 and 2,
every request of config 4), so it is itself held to the oracle here, on the same seeded inputs.
"""

import numpy as np
import pytest

import cpu_native
from cpu_sim import CpuSim, stable_topk
from pto_wsp_b200 import workloads


@pytest.mark.parametrize("kind", ["rmsnorm", "softmax"])
def test_row_tiles_match_the_oracle(kind):
    rng = np.random.default_rng(5)
    B, T, R, C = (2, 8, 16, 128) if kind == "rmsnorm" else (2, 4, 32, 256)
    x = rng.standard_normal((B, T, R, C), dtype=np.float32) * (4 if kind == "softmax" else 1)
    if kind == "softmax":
        x[rng.random(x.shape) < 0.01] = 30.0
    plan = (workloads.rmsnorm_plan if kind == "rmsnorm" else workloads.softmax_plan)(B, T, R, C)
    want = np.zeros_like(x)
    CpuSim(plan).run([x, want])
    got = np.zeros_like(x)
    cpu_native.row_tiles(kind, x, got, R, C, 3)
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-9)


def test_gemm_tiles_match_the_oracle():
    rng = np.random.default_rng(6)
    B, M, N, K = 2, 256, 256, 128
    a = rng.uniform(-1, 1, (B, M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (B, K, N)).astype(np.float16)
    want = np.zeros((B, M, N), np.float32)
    CpuSim(workloads.bgemm_plan(B, M, N, K)).run(list(workloads.bgemm_views(a, b, want)))
    got = np.zeros_like(want)
    cpu_native.gemm_tiles(a, b, got, 128, 128, 3)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)


def test_paged_decode_matches_the_oracle():
    rng = np.random.default_rng(7)
    lengths = [0, 1, 16, 17, 300, 513]
    plan, arrays = workloads.decode_inputs(rng, len(lengths), lengths=lengths)
    want = [a.copy() for a in arrays]
    CpuSim(plan).run(want, axis_sizes={"b": len(lengths)})
    q, kc, vc, pt, kl, _ = arrays
    got = np.zeros_like(arrays[5])
    cpu_native.paged_decode(q, kc, vc, pt, kl, got, 16, 3)
    ref = want[5].astype(np.float64)
    err = np.abs(got.astype(np.float64) - ref)
    assert np.all(err <= 2e-3 * np.abs(ref) + 2e-3), float(err.max())
    assert not got[0].any()  # an empty request writes zeros


def test_indexer_scores_and_stable_topk():
    rng = np.random.default_rng(8)
    B, T, K = 1, 1024, 64
    plan, arrays = workloads.indexer_inputs(rng, B, T, K)
    want = [a.copy() for a in arrays]
    CpuSim(plan).run(want)
    q, k, w = arrays[:3]
    s = np.zeros_like(arrays[3])
    idx = np.zeros_like(arrays[4])
    cpu_native.indexer(q, k, w, s, idx, 64, 3)
    ref = want[3].astype(np.float64)
    assert np.max(np.abs(s - ref) / (np.abs(ref) + np.abs(ref).mean())) < 1e-4
    for row in range(s.shape[1]):  # the port's indices are the stable top-k of the port's own scores
        np.testing.assert_array_equal(idx[0, row], stable_topk(s[0, row], K))
