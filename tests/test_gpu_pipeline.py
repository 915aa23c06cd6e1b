"""Overlapped host-staged runs (-m gpu).

A static single-batch workload whose host tensors hold 64 MiB or more runs as
chunks of tasks whose host->device copies, kernels and device->host copies
overlap on three streams.  Its results must be bit-identical to the serial
run (`pipeline_chunks` = 1): same kernels on the same rows, only the copies
are cut differently.  Each input byte is copied in once and each output byte
comes back at least once, whatever order the task loop visits memory in.
"""

import numpy as np
import pytest

from pto_wsp_b200 import workloads
from pto_wsp_b200.runtime import CudaExecutable

pytestmark = pytest.mark.gpu


def run(plan, x, chunks, y=None):
    ex = CudaExecutable(plan)
    ex.set_option("pipeline_chunks", chunks)
    if y is None:
        y = np.full_like(x, np.nan)
    cycles = ex.run_with_symbols([x, y], {}, {}, {})
    return cycles, y, ex.timing()


@pytest.mark.parametrize("kind", ["softmax", "rmsnorm"])
def test_pipelined_matches_serial(kind, require_cuda):
    rng = np.random.default_rng(3)
    if kind == "softmax":
        plan = workloads.softmax_plan(2, 1024)  # 2 x 1024 tiles of 32 x 256 f32: 64 MiB in, 64 MiB out
        x = rng.standard_normal((2, 1024, 32, 256), dtype=np.float32) * 3
    else:
        plan = workloads.rmsnorm_plan(4, 1024)  # 4 x 1024 tiles of 16 x 128 f32: 32 MiB in, 32 MiB out
        x = rng.standard_normal((4, 1024, 16, 128), dtype=np.float32)
    c1, y1, t1 = run(plan, x, 1)
    c16, y16, t16 = run(plan, x, 16)
    assert c1 == c16
    assert np.array_equal(y1, y16)
    assert t1["h2d_bytes"] == x.nbytes and t1["d2h_bytes"] == x.nbytes
    assert t16["h2d_bytes"] == x.nbytes and t16["d2h_bytes"] == x.nbytes  # copied once each way
    assert t16["launches"] == 16 and t1["launches"] == 1


def test_pipelined_pinned_and_repeat(require_cuda):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(4)
    plan = workloads.softmax_plan(4, 512)
    xt = torch.empty((4, 512, 32, 256), dtype=torch.float32, pin_memory=True)
    yt = torch.empty_like(xt).pin_memory()
    x = xt.numpy()
    x[...] = rng.standard_normal(x.shape, dtype=np.float32)
    _, y_ref, _ = run(plan, x, 1)
    ex = CudaExecutable(plan)
    xd = torch.from_numpy(x).cuda()  # first run device-resident: its cached task table is then reused below
    yd = torch.empty_like(xd)
    ex.run_with_symbols([xd, yd], {}, {}, {})
    assert ex.timing()["launches"] == 1
    for _ in range(3):  # second and third runs replay the cached task table
        yt.fill_(float("nan"))
        ex.run_with_symbols([x, yt.numpy()], {}, {}, {})
        assert np.array_equal(yt.numpy(), y_ref)
        assert ex.timing()["launches"] > 1


def test_pipelined_interleaved_layout(require_cuda):
    # Memory order [T, B, rows, cols] while the task loop runs b outer, t inner:
    # every chunk's range spans most of both tensors.  Inputs are still copied
    # once; overlapping output ranges come back in chunk order, so the last
    # copy of each element is taken after the task that writes it.
    rng = np.random.default_rng(5)
    B, T = 2, 2048
    plan = workloads.softmax_plan(B, T)
    xs = rng.standard_normal((T, B, 32, 256), dtype=np.float32).transpose(1, 0, 2, 3)
    ys = np.full((T, B, 32, 256), np.nan, np.float32).transpose(1, 0, 2, 3)
    _, y1, _ = run(plan, np.ascontiguousarray(xs), 1)
    c, y, t = run(plan, xs, 16, ys)
    assert np.array_equal(np.ascontiguousarray(y), y1)
    assert t["h2d_bytes"] == xs.nbytes
    assert t["d2h_bytes"] >= xs.nbytes


def test_pipelined_bgemm(require_cuda):
    # tcgen05 matmul batches pipeline from their second host-staged run (the first checks the layout); each chunk
    # runs the one-CTA tile kernel on its own tasks, so results agree with the serial run's CTA-pair launch
    rng = np.random.default_rng(6)
    B, M, N, K = 8, 1024, 1024, 1024  # 16 + 16 MiB f16 in, 32 MiB f32 out
    plan = workloads.bgemm_plan(B, M, N, K)
    a = (rng.random((B, M, K), dtype=np.float32) * 2 - 1).astype(np.float16)
    b = (rng.random((B, K, N), dtype=np.float32) * 2 - 1).astype(np.float16)
    c1 = np.full((B, M, N), np.nan, np.float32)
    ex1 = CudaExecutable(plan)
    ex1.set_option("pipeline_chunks", 1)
    cyc1 = ex1.run_with_symbols(list(workloads.bgemm_views(a, b, c1)), {}, {}, {})
    ex = CudaExecutable(plan)
    ex.set_option("pipeline_chunks", 16)
    for i in range(2):
        c = np.full((B, M, N), np.nan, np.float32)
        assert ex.run_with_symbols(list(workloads.bgemm_views(a, b, c)), {}, {}, {}) == cyc1
        t = ex.timing()
        assert t["h2d_bytes"] == a.nbytes + b.nbytes and t["d2h_bytes"] == c.nbytes
        assert (t["launches"] == 16) == (i == 1)  # pipelined once the layout check has run
        assert t["chunks"] == (16 if i == 1 else 0)
        np.testing.assert_allclose(c, c1, rtol=1e-5, atol=1e-5)
    ref = a[0].astype(np.float64) @ b[0].astype(np.float64)
    assert np.max(np.abs(c[0] - ref) / (np.abs(ref) + np.sqrt(np.mean(ref ** 2)))) < 2e-3


def test_pipelined_indexer_chain(require_cuda):
    # two waves (scoring, then top-k over the scores) run chunk by chunk: chunk c's top-k reads the scores chunk c
    # just wrote; the scores are never staged in (written before they are read) and both outputs come back
    rng = np.random.default_rng(7)
    plan, arrays = workloads.indexer_inputs(rng, 8, 32768, 2048)  # 64 MiB of keys
    serial = [a.copy() for a in arrays]
    ex1 = CudaExecutable(plan)
    ex1.set_option("pipeline_chunks", 1)
    cyc1 = ex1.run_with_symbols(serial, {}, {}, {})
    ex = CudaExecutable(plan)
    ex.set_option("pipeline_chunks", 16)
    for i in range(2):
        got = [a.copy() for a in arrays]
        got[3][...] = np.nan
        got[4][...] = -1
        assert ex.run_with_symbols(got, {}, {}, {}) == cyc1
        t = ex.timing()
        assert t["h2d_bytes"] == sum(a.nbytes for a in arrays[:3])
        assert t["d2h_bytes"] == arrays[3].nbytes + arrays[4].nbytes
        assert (t["launches"] == 16) == (i == 1)  # 8 chunks x (scoring, top-k) once the layout check has run
        assert t["chunks"] == (8 if i == 1 else 0)
        np.testing.assert_allclose(got[3], serial[3], rtol=1e-6, atol=1e-6)
        assert np.array_equal(got[4], serial[4])
