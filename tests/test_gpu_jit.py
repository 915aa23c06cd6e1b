"""Fused row kernels of generic tile programs vs the oracle (-m gpu).

Element-wise ops and max reductions are bit-exact against the oracle (the
same IEEE operations in the same order); sum reductions add in tree order,
so RMSNorm / softmax of odd widths are checked with the 1e-5 fp32 bar.
"""

import numpy as np
import pytest
from cpu_sim import CpuSim
from test_jit import long_chain_plan, rowmax_shift_plan

from pto_wsp_b200 import workloads
from pto_wsp_b200.runtime import CudaExecutable

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cols,dtype", [(40, "f32"), (96, "f16"), (600, "f32"), (1, "f32"), (4, "f32"), (12, "f16"), (200, "f16"), (1024, "f32")])
def test_generic_row_kernel_bit_exact(cols, dtype, require_cuda):
    rng = np.random.default_rng(cols)
    B, T, R = 3, 5, 8
    plan = rowmax_shift_plan(B, T, R, cols, dtype)
    x = rng.standard_normal((B, T, R, cols)).astype(np.float16 if dtype == "f16" else np.float32)
    y = rng.standard_normal((B, T, R, cols)).astype(np.float32)
    ref = np.full((B, T, R, cols), np.nan, np.float32)
    cyc = CpuSim(plan).run([x, y, ref])
    got = np.full_like(ref, np.nan)
    ex = CudaExecutable(plan)
    assert ex.run_with_symbols([x, y, got], {}, {}, {}) == cyc
    assert ex.describe()["kernels"][0]["row_kernel"] == "loaded"
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("kind,cols", [("rmsnorm", 96), ("softmax", 200), ("softmax", 33)])
def test_row_ops_of_odd_widths_run_fused(kind, cols, require_cuda):
    rng = np.random.default_rng(7)
    B, T, R = 4, 16, 16
    plan = (workloads.rmsnorm_plan if kind == "rmsnorm" else workloads.softmax_plan)(B, T, R, cols)
    x = (rng.standard_normal((B, T, R, cols)) * 3).astype(np.float32)
    ref = np.zeros_like(x)
    cyc = CpuSim(plan).run([x, ref])
    got = np.full_like(x, np.nan)
    ex = CudaExecutable(plan)
    assert ex.run_with_symbols([x, got], {}, {}, {}) == cyc
    assert ex.describe()["kernels"][0]["row_kernel"] == "loaded"  # the fast path does not take this width
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-7)


def col_scale_plan(B, R, C, dtype_x="f32"):
    """out = (x - v) * w with v, w one-row [1, C] operands (column broadcasts) and x [R, C]."""
    from pto_wsp_b200.workloads import KernelBuilder, _pfor, _plan, _schedule, _targ, _task

    k = KernelBuilder("col_scale")
    x = k.param("x", dtype_x, R, C)
    v = k.param("v", "f32", 1, C)
    w = k.param("w", "f32", 1, C)
    out = k.param("out", "f32", R, C)
    d = k.op("Sub", [x, v], ("f32", R, C))
    k.store(out, k.op("Mul", [d, w], ("f32", R, C)))
    body = _pfor("b", B, _task("col_scale", ["b"], [_targ("x", 0, 3, ["b"]), _targ("v", 1, 3, ["b"]),
                                                   _targ("w", 2, 3, ["b"]), _targ("out", 3, 3, ["b"])]))
    return _plan("col_scale", [(dtype_x, [B, R, C]), ("f32", [B, 1, C]), ("f32", [B, 1, C]), ("f32", [B, R, C])],
                 [k.build()], body, _schedule())


@pytest.mark.parametrize("cols,dtype", [(64, "f32"), (36, "f16"), (33, "f32"), (1000, "f32")])
def test_column_broadcast_row_kernel_bit_exact(cols, dtype, require_cuda):
    rng = np.random.default_rng(cols + 1)
    B, R = 6, 16
    plan = col_scale_plan(B, R, cols, dtype)
    x = rng.standard_normal((B, R, cols)).astype(np.float16 if dtype == "f16" else np.float32)
    v = rng.standard_normal((B, 1, cols)).astype(np.float32)
    w = rng.standard_normal((B, 1, cols)).astype(np.float32)
    ref = np.full((B, R, cols), np.nan, np.float32)
    cyc = CpuSim(plan).run([x, v, w, ref])
    got = np.full_like(ref, np.nan)
    ex = CudaExecutable(plan)
    assert ex.run_with_symbols([x, v, w, got], {}, {}, {}) == cyc
    assert ex.describe()["kernels"][0]["row_kernel"] == "loaded"
    np.testing.assert_array_equal(got, ref)


def row_vector_plan(B, R, C):
    """out = (x + v) * v with v a one-row [1, R] operand: the emitter's row broadcast (element r to row r)."""
    from pto_wsp_b200.workloads import KernelBuilder, _pfor, _plan, _schedule, _targ, _task

    k = KernelBuilder("row_vec")
    x = k.param("x", "f32", R, C)
    v = k.param("v", "f32", 1, R)
    out = k.param("out", "f32", R, C)
    d = k.op("Add", [x, v], ("f32", R, C))
    k.store(out, k.op("Mul", [d, v], ("f32", R, C)))
    body = _pfor("b", B, _task("row_vec", ["b"], [_targ("x", 0, 3, ["b"]), _targ("v", 1, 3, ["b"]),
                                                 _targ("out", 2, 3, ["b"])]))
    return _plan("row_vec", [("f32", [B, R, C]), ("f32", [B, 1, R]), ("f32", [B, R, C])], [k.build()], body,
                 _schedule())


@pytest.mark.parametrize("R,C", [(16, 64), (8, 40), (32, 33)])
def test_one_row_operand_broadcast_over_rows_bit_exact(R, C, require_cuda):
    rng = np.random.default_rng(R * C)
    B = 5
    plan = row_vector_plan(B, R, C)
    x = rng.standard_normal((B, R, C)).astype(np.float32)
    v = rng.standard_normal((B, 1, R)).astype(np.float32)
    ref = np.full((B, R, C), np.nan, np.float32)
    cyc = CpuSim(plan).run([x, v, ref])
    got = np.full_like(ref, np.nan)
    ex = CudaExecutable(plan)
    assert ex.run_with_symbols([x, v, got], {}, {}, {}) == cyc
    assert ex.describe()["kernels"][0]["row_kernel"] == "loaded"
    np.testing.assert_array_equal(got, ref)


def test_long_op_chain_bit_exact(require_cuda):
    rng = np.random.default_rng(9)
    plan = long_chain_plan(5, 8, 96)
    x = rng.standard_normal((5, 8, 96)).astype(np.float32)
    ref = np.full_like(x, np.nan)
    cyc = CpuSim(plan).run([x, ref])
    got = np.full_like(x, np.nan)
    ex = CudaExecutable(plan)
    assert ex.run_with_symbols([x, got], {}, {}, {}) == cyc
    assert ex.describe()["kernels"][0]["row_kernel"] == "loaded"
    np.testing.assert_array_equal(got, ref)
