"""bgemm on tcgen05 vs the oracle and an fp64 recompute (-m gpu).

Tolerance (north_star): fp16 contractions within 2e-3 relative of an fp64
recompute -- checked element-wise as a plain relative error on every element
with |C64| >= 1e-2 rms(C64) (smaller ones: absolute 2e-3 x that floor).  At
full size all 64 batch elements are recomputed in fp64 on the GPU.
"""

import numpy as np
import pytest
from cpu_sim import CpuSim

from tolerance import RTOL_F16_MMA, assert_rel, rms

from pto_wsp_b200 import workloads
from pto_wsp_b200.runtime import CudaExecutable

pytestmark = pytest.mark.gpu


def check(c, ref):
    return assert_rel(c, ref, RTOL_F16_MMA, 1e-2 * rms(ref))


def inputs(rng, B, M, N, K):
    a = rng.uniform(-1, 1, (B, M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (B, K, N)).astype(np.float16)
    return a, b


@pytest.mark.parametrize("B,M,N,K", [(2, 256, 256, 512), (1, 128, 128, 64), (3, 384, 128, 1024)])
def test_bgemm_tcgen05_vs_oracle(B, M, N, K, require_cuda):
    rng = np.random.default_rng(0)
    a, b = inputs(rng, B, M, N, K)
    plan = workloads.bgemm_plan(B, M, N, K)
    c_ref = np.zeros((B, M, N), np.float32)
    cyc_ref = CpuSim(plan).run(list(workloads.bgemm_views(a, b, c_ref)))
    c = np.zeros((B, M, N), np.float32)
    ex = CudaExecutable(plan)
    assert ex.describe()["kernels"][0]["impl"] == "matmul_tcgen05"
    assert ex.run_with_symbols(list(workloads.bgemm_views(a, b, c)), {}, {}, {}) == cyc_ref
    check(c, a.astype(np.float64) @ b.astype(np.float64))
    check(c, c_ref)


def test_bgemm_accumulate_form(require_cuda):
    rng = np.random.default_rng(1)
    B, M, N, K = 2, 256, 256, 256
    a, b = inputs(rng, B, M, N, K)
    c0 = rng.standard_normal((B, M, N)).astype(np.float32)
    plan = workloads.bgemm_plan(B, M, N, K, accumulate=True)
    c = c0.copy()
    ex = CudaExecutable(plan)
    assert ex.describe()["kernels"][0]["impl"] == "matmul_tcgen05_acc"
    ex.run_with_symbols(list(workloads.bgemm_views(a, b, c)), {}, {}, {})
    check(c, c0.astype(np.float64) + a.astype(np.float64) @ b.astype(np.float64))


@pytest.mark.parametrize("tn", [64, 256])
def test_bgemm_other_tile_widths(tn, require_cuda):
    rng = np.random.default_rng(2)
    B, M, N, K = 1, 256, 512, 192
    a, b = inputs(rng, B, M, N, K)
    plan = workloads.bgemm_plan(B, M, N, K, tile_n=tn)
    c = np.zeros((B, M, N), np.float32)
    CudaExecutable(plan).run_with_symbols(list(workloads.bgemm_views(a, b, c, tile_n=tn)), {}, {}, {})
    check(c, a.astype(np.float64) @ b.astype(np.float64))


def test_bgemm_config3_full_size(require_cuda):
    torch = pytest.importorskip("torch")
    B, M, N, K = 64, 2048, 2048, 2048
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    a = (torch.rand((B, M, K), generator=g, device="cuda") * 2 - 1).half()
    b = (torch.rand((B, K, N), generator=g, device="cuda") * 2 - 1).half()
    c = torch.full((B, M, N), float("nan"), device="cuda")
    ex = CudaExecutable(workloads.bgemm_plan(B, M, N, K))
    ex.run_with_symbols(list(workloads.bgemm_views(a, b, c)), {}, {}, {})
    assert not torch.isnan(c).any()
    worst = 0.0
    for b0 in range(0, B, 8):  # every batch element, recomputed in fp64 on the GPU, 8 at a time
        ref = torch.bmm(a[b0:b0 + 8].double(), b[b0:b0 + 8].double())
        floor = 1e-2 * float(ref.pow(2).mean().sqrt())
        err = (c[b0:b0 + 8].double() - ref).abs()
        big = ref.abs() >= floor
        rel = float((err[big] / ref.abs()[big]).max())
        assert rel <= RTOL_F16_MMA, (b0, rel)
        assert float(err[~big].max()) <= RTOL_F16_MMA * floor if bool((~big).any()) else True
        worst = max(worst, rel)
        del ref, err, big
    print(f"bgemm config 3: worst relative error over all 64 batch elements {worst:.3g}")
