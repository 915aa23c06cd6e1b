"""bgemm on tcgen05 vs the oracle and an fp64 recompute (-m gpu).

Tolerance (north_star): fp16 contractions within 2e-3 relative of an fp64
recompute -- checked element-wise as |C - C64| <= 2e-3 * (|C64| + rms(C64)).
"""

import numpy as np
import pytest
from cpu_sim import CpuSim

from pto_wsp_b200 import workloads
from pto_wsp_b200.runtime import CudaExecutable

pytestmark = pytest.mark.gpu
RTOL = 2e-3


def check(c, ref):
    ref = np.asarray(ref, np.float64)
    scale = np.sqrt(np.mean(ref * ref)) + 1e-30
    err = np.abs(np.asarray(c, np.float64) - ref)
    assert np.all(err <= RTOL * (np.abs(ref) + scale)), float((err / (np.abs(ref) + scale)).max())


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
    for bi in (0, 37, 63):
        ref = (a[bi].double() @ b[bi].double()).cpu().numpy()
        check(c[bi].cpu().numpy(), ref)
    assert not torch.isnan(c).any()
