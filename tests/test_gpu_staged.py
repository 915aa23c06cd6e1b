"""Generic kernels cut at their contractions (-m gpu): matmul stages (tcgen05 for f16 tiles of its shapes, CUDA-core
fused multiply-adds otherwise) and fused row programs, with the values between them in HBM scratch.  The f32 MLP's
stages do the tile program's arithmetic in its order, so it matches the oracle bit for bit; the attention kernel's
first contraction runs on tensor cores and is held to the f16-contraction tolerance, 2e-3 relative."""

import numpy as np
import pytest
from _staged import attention_arrays, attention_plan, inout_plan, mlp_arrays, mlp_plan
from cpu_sim import CpuSim

from pto_wsp_b200.runtime import CudaExecutable

pytestmark = pytest.mark.gpu


def test_f32_mlp_stages_bit_exact(require_cuda):
    rng = np.random.default_rng(11)
    T, rows, d, hidden = 6, 64, 512, 256  # x tile 128 KB, W1 512 KB: far beyond one CTA's shared memory
    plan = mlp_plan(T, rows, d, hidden)
    arrays = mlp_arrays(rng, T, rows, d, hidden)
    ref = [a.copy() for a in arrays]
    cyc = CpuSim(plan).run(ref)
    ex = CudaExecutable(plan)
    k = ex.describe()["kernels"][0]
    assert k["impl"] == "staged_matmul+row_programs"
    assert k["stages"] == ["matmul 64x256x512 cuda_cores", "rows 64", "matmul 64x512x256 cuda_cores", "rows 64"]
    for _ in range(2):  # the second run replays the cached task table and stage records
        got = [a.copy() for a in arrays]
        assert ex.run_with_symbols(got, {}, {}, {}) == cyc
        assert np.array_equal(got[3], ref[3])
    assert ex.timing()["launches"] == 4
    torch = pytest.importorskip("torch")
    dev = [torch.from_numpy(a.copy()).cuda() for a in arrays]
    ex.run_with_symbols(dev, {}, {}, {})
    assert np.array_equal(dev[3].cpu().numpy(), ref[3])
    # a 1 MiB scratch budget: 256 KB of crossing values per task, so the stages run over groups of 4 tasks
    ex = CudaExecutable(plan)
    ex.set_option("stage_scratch_mb", 1)
    got = [a.copy() for a in arrays]
    assert ex.run_with_symbols(got, {}, {}, {}) == cyc
    assert np.array_equal(got[3], ref[3])
    assert ex.timing()["launches"] == 8  # groups of 4 and 2 tasks x 4 stages


@pytest.mark.parametrize("B,H,QT,kv_len,first", [
    (2, 3, 2, 256, "matmul 128x256x128 tcgen05"),
    (2, 3, 2, 128, "matmul 128x128x128 tcgen05"),
    (1, 2, 1, 1024, "matmul 128x1024x128 tcgen05 (4 tiles of 256)"),  # each task's scores as four 128 x 256 tiles
])
def test_attention_stages_vs_oracle(B, H, QT, kv_len, first, require_cuda):
    rng = np.random.default_rng(kv_len)
    plan = attention_plan(B, H, QT, kv_len)
    arrays = attention_arrays(rng, B, H, QT, kv_len)
    ref = [a.copy() for a in arrays]
    cyc = CpuSim(plan).run(ref)
    ex = CudaExecutable(plan)
    ex.set_option("fused_attention", 0)  # the staged form (the fused kernel has tests/test_gpu_attention.py)
    k = ex.describe()["kernels"][0]
    assert k["stages"][0] == first
    assert k["stages"][2] == f"matmul 128x128x{kv_len} cuda_cores"
    got = [a.copy() for a in arrays]
    assert ex.run_with_symbols(got, {}, {}, {}) == cyc
    o, r = got[3].astype(np.float64), ref[3].astype(np.float64)
    scale = np.sqrt(np.mean(r * r))
    assert np.all(np.abs(o - r) <= 2e-3 * (np.abs(r) + scale)), float((np.abs(o - r) / (np.abs(r) + scale)).max())
    # fp64 recompute of one tile: softmax(scale * q . k^T) . v
    b, h, qt = B - 1, H - 1, QT - 1
    q = arrays[0][b, h, qt].astype(np.float64)
    kt = arrays[1][b, h].astype(np.float64)
    v = arrays[2][b, h].astype(np.float64)
    s = (q @ kt) * np.float64(np.float32(0.088))
    w = np.exp(s - s.max(axis=1, keepdims=True))
    w /= w.sum(axis=1, keepdims=True)
    o64 = w @ v
    assert np.all(np.abs(got[3][b, h, qt] - o64) <= 2e-3 * (np.abs(o64) + np.sqrt(np.mean(o64 * o64))))
    if kv_len >= 1024:
        # a 1 MiB scratch budget: the stages run over groups of tasks, the tcgen05 stage's records and the
        # scratch offsets repeating per group; same kernels, same data -> the same bits as one group
        small = CudaExecutable(plan)
        small.set_option("fused_attention", 0)  # the stages themselves, not the fused kernel
        small.set_option("stage_scratch_mb", 1)
        again = [a.copy() for a in arrays]
        assert small.run_with_symbols(again, {}, {}, {}) == cyc
        assert small.timing()["launches"] > 4  # four stages, more than one group of tasks
        staged = CudaExecutable(plan)
        staged.set_option("fused_attention", 0)
        once = [a.copy() for a in arrays]
        staged.run_with_symbols(once, {}, {}, {})
        assert np.array_equal(again[3], once[3])  # one group or several: the same bits


def test_param_stored_before_a_later_stage_reads_its_old_value(require_cuda):
    # p is doubled in the first row stage; the last stage adds the old p, kept in scratch (not re-read)
    rng = np.random.default_rng(5)
    plan = inout_plan(3)
    arrays = [rng.standard_normal((3, 128, 128)).astype(np.float32) for _ in range(3)]
    arrays.append(np.full((3, 128, 128), np.nan, np.float32))
    ref = [a.copy() for a in arrays]
    cyc = CpuSim(plan).run(ref)
    ex = CudaExecutable(plan)
    assert ex.describe()["kernels"][0]["scratch_tiles"] == 2
    got = [a.copy() for a in arrays]
    assert ex.run_with_symbols(got, {}, {}, {}) == cyc
    assert np.array_equal(got[0], ref[0]) and np.array_equal(got[3], ref[3])
