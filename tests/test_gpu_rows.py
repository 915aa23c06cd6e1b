"""RMSNorm and softmax row kernels vs the oracle (-m gpu).

Tolerance (north_star): fp32 row ops within 1e-5 relative of the reference;
here against the CPU oracle (reference op order) and an fp64 recompute.
"""

import numpy as np
import pytest
from cpu_sim import CpuSim

from pto_wsp_b200 import workloads
from pto_wsp_b200.runtime import CudaExecutable

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def rms64(x):
    x = x.astype(np.float64)
    return x / np.sqrt((x * x).mean(-1, keepdims=True))


def softmax64(x):
    x = x.astype(np.float64)
    e = np.exp(x - x.max(-1, keepdims=True))
    return e / e.sum(-1, keepdims=True)


def softmax_input(rng, shape):
    x = (rng.standard_normal(shape, dtype=np.float32) * 4.0).astype(np.float32)
    x[rng.random(shape) < 0.01] = 30.0
    return x


@pytest.mark.parametrize("B,T", [(4, 64), (1, 1), (3, 5)])
def test_rmsnorm_config1_vs_oracle(B, T, require_cuda):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((B, T, 16, 128), dtype=np.float32)
    plan = workloads.rmsnorm_plan(B, T)
    y_ref = np.zeros_like(x)
    c_ref = CpuSim(plan).run([x, y_ref])
    y = np.zeros_like(x)
    ex = CudaExecutable(plan)
    assert ex.describe()["kernels"][0]["impl"] == "rmsnorm_rows"
    assert ex.run_with_symbols([x, y], {}, {}, {}) == c_ref
    np.testing.assert_allclose(y, y_ref, rtol=RTOL, atol=1e-7)
    np.testing.assert_allclose(y, rms64(x), rtol=RTOL, atol=1e-7)


@pytest.mark.parametrize("B,T,R,C", [(2, 16, 32, 256), (1, 3, 32, 128), (2, 2, 8, 512), (1, 2, 4, 1024)])
def test_softmax_vs_oracle(B, T, R, C, require_cuda):
    rng = np.random.default_rng(1)
    x = softmax_input(rng, (B, T, R, C))
    plan = workloads.softmax_plan(B, T, R, C)
    y_ref = np.zeros_like(x)
    c_ref = CpuSim(plan).run([x, y_ref])
    y = np.zeros_like(x)
    ex = CudaExecutable(plan)
    assert ex.run_with_symbols([x, y], {}, {}, {}) == c_ref
    np.testing.assert_allclose(y, y_ref, rtol=RTOL, atol=1e-30)
    np.testing.assert_allclose(y, softmax64(x), rtol=RTOL, atol=1e-30)


@pytest.mark.parametrize("C", [96, 200])
def test_row_ops_with_odd_widths_run_the_nvrtc_row_program(C, require_cuda):
    rng = np.random.default_rng(2)
    x = softmax_input(rng, (2, 3, 8, C))
    plan = workloads.softmax_plan(2, 3, 8, C)
    y = np.zeros_like(x)
    ex = CudaExecutable(plan)
    ex.run_with_symbols([x, y], {}, {}, {})
    np.testing.assert_allclose(y, softmax64(x), rtol=RTOL, atol=1e-30)
    assert ex.describe()["kernels"][0].get("row_kernel") == "loaded"


def test_device_resident_tensors_run_in_place(require_cuda):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(3)
    x = softmax_input(rng, (2, 8, 32, 256))
    xd = torch.from_numpy(x).cuda()
    yd = torch.zeros_like(xd)
    ex = CudaExecutable(workloads.softmax_plan(2, 8))
    ex.run_with_symbols([xd, yd], {}, {}, {})
    t = ex.timing()
    assert t["h2d_bytes"] == 0 and t["d2h_bytes"] == 0 and t["launches"] == 1
    np.testing.assert_allclose(yd.cpu().numpy(), softmax64(x), rtol=RTOL, atol=1e-30)


def test_write_only_output_is_not_staged_in(require_cuda):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 4, 16, 128), dtype=np.float32)
    y = np.full_like(x, np.nan)
    ex = CudaExecutable(workloads.rmsnorm_plan(2, 4))
    ex.run_with_symbols([x, y], {}, {}, {})
    t = ex.timing()
    assert t["h2d_bytes"] == x.nbytes and t["d2h_bytes"] == y.nbytes
    np.testing.assert_allclose(y, rms64(x), rtol=RTOL, atol=1e-7)


@pytest.mark.parametrize("workload", ["softmax", "rmsnorm"])
def test_full_size_config_properties(workload, require_cuda):
    """BASELINE sizes: rows sum to 1 / have unit mean square, checked on-device (size-independent properties)."""
    torch = pytest.importorskip("torch")
    if workload == "softmax":
        B, T, R, C = 32, 2048, 32, 256
        plan = workloads.softmax_plan(B, T)
    else:
        B, T, R, C = 64, 4096, 16, 128
        plan = workloads.rmsnorm_plan(B, T)
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    x = torch.randn((B, T, R, C), generator=g, device="cuda")
    if workload == "softmax":
        x *= 4.0
        x[torch.rand(x.shape, generator=g, device="cuda") < 0.01] = 30.0
    y = torch.empty_like(x)
    CudaExecutable(plan).run_with_symbols([x, y], {}, {}, {})
    if workload == "softmax":
        s = y.double().sum(-1)
        assert torch.allclose(s, torch.ones_like(s), rtol=0, atol=2e-5)
        assert bool((y >= 0).all())
    else:
        ms = (y.double() ** 2).mean(-1)
        assert torch.allclose(ms, torch.ones_like(ms), rtol=0, atol=2e-5)
    # sampled tiles against fp64
    idx = torch.randint(0, B * T, (64,), generator=g, device="cuda")
    xs = x.reshape(B * T, R, C)[idx].cpu().numpy()
    ys = y.reshape(B * T, R, C)[idx].cpu().numpy()
    ref = softmax64(xs) if workload == "softmax" else rms64(xs)
    np.testing.assert_allclose(ys, ref, rtol=RTOL, atol=1e-30 if workload == "softmax" else 1e-7)
    # every tile against the C port of the CPU-sim task (reference op order, all host threads), 1e-5 relative
    import cpu_native

    xh, yh = x.reshape(B * T, R, C).cpu().numpy(), y.reshape(B * T, R, C).cpu().numpy()
    del x, y
    torch.cuda.empty_cache()
    port = np.empty_like(xh)
    cpu_native.row_tiles(workload, xh, port, R, C)
    for t0 in range(0, B * T, 8192):
        np.testing.assert_allclose(yh[t0:t0 + 8192], port[t0:t0 + 8192], rtol=RTOL,
                                   atol=1e-30 if workload == "softmax" else 1e-7)
