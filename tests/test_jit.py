"""Row-program compiler, host side (no GPU needed).

Generic row-local kernels (element-wise ops, row broadcasts, row reductions
over whole tiles) get a fused kernel built with NVRTC when the program is
compiled; other kernels keep the tile-program interpreter and say why.
"""

import pytest

from pto_wsp_b200 import workloads
from pto_wsp_b200.runtime import CudaExecutable
from pto_wsp_b200.workloads import KernelBuilder, _pfor, _plan, _schedule, _targ, _task


def rowmax_shift_plan(B, T, R, C, dtype_x="f32"):
    """out = (x - rowmax(x)) * y: element-wise ops, a row reduction and a row broadcast."""
    k = KernelBuilder("shift_scale")
    x = k.param("x", dtype_x, R, C)
    y = k.param("y", "f32", R, C)
    out = k.param("out", "f32", R, C)
    m = k.op("RowMax", [x], ("f32", R, 1))
    d = k.op("Sub", [x, m], ("f32", R, C))
    p = k.op("Mul", [d, y], ("f32", R, C))
    k.store(out, p)
    body = _pfor("b", B, _pfor("h", T, _task("shift_scale", ["b", "h"], [
        _targ("x", 0, 4, ["b", "h"]), _targ("y", 1, 4, ["b", "h"]), _targ("out", 2, 4, ["b", "h"])])))
    return _plan("shift_scale", [(dtype_x, [B, T, R, C]), ("f32", [B, T, R, C]), ("f32", [B, T, R, C])],
                 [k.build()], body, _schedule())


def nvrtc_available() -> bool:
    return CudaExecutable(rowmax_shift_plan(1, 1, 4, 40)).describe()["kernels"][0]["row_kernel_note"] != "NVRTC not found"


@pytest.mark.parametrize("cols,dtype", [(40, "f32"), (96, "f16"), (1000, "f32"), (1, "f32")])
def test_generic_row_kernels_compile(cols, dtype):
    if not nvrtc_available():
        pytest.skip("NVRTC not installed")
    d = CudaExecutable(rowmax_shift_plan(2, 3, 8, cols, dtype)).describe()["kernels"][0]
    assert d["impl"] == "tile_program"
    assert d["row_kernel"] == "compiled", d["row_kernel_note"]


def col_broadcast_plan(R, C):
    k = KernelBuilder("sub_col")
    x = k.param("x", "f32", R, C)
    v = k.param("v", "f32", 1, C)
    out = k.param("out", "f32", R, C)
    k.store(out, k.op("Sub", [x, v], ("f32", R, C)))
    body = _pfor("b", 2, _task("sub_col", ["b"], [_targ("x", 0, 3, ["b"]), _targ("v", 1, 3, ["b"]),
                                                   _targ("out", 2, 3, ["b"])]))
    return _plan("sub_col", [("f32", [2, R, C]), ("f32", [2, 1, C]), ("f32", [2, R, C])], [k.build()], body,
                 _schedule())


def col_store_plan(R, C):
    """A many-row program that also stores a one-row tile: every row would write it, so it stays interpreted."""
    k = KernelBuilder("col_store")
    x = k.param("x", "f32", R, C)
    v = k.param("v", "f32", 1, C)
    out = k.param("out", "f32", R, C)
    vo = k.param("vo", "f32", 1, C)
    k.store(out, k.op("Sub", [x, v], ("f32", R, C)))
    k.store(vo, k.op("Mul", [v, v], ("f32", 1, C)))
    body = _pfor("b", 2, _task("col_store", ["b"], [_targ("x", 0, 3, ["b"]), _targ("v", 1, 3, ["b"]),
                                                     _targ("out", 2, 3, ["b"]), _targ("vo", 3, 3, ["b"])]))
    return _plan("col_store", [("f32", [2, R, C]), ("f32", [2, 1, C]), ("f32", [2, R, C]), ("f32", [2, 1, C])],
                 [k.build()], body, _schedule())


def test_column_broadcasts_are_row_local():
    d = CudaExecutable(col_broadcast_plan(4, 64)).describe()["kernels"][0]
    assert d["impl"] == "tile_program" and d["row_kernel"] == "compiled", d["row_kernel_note"]


def test_kernels_outside_the_row_local_set_keep_the_interpreter():
    d = CudaExecutable(col_store_plan(4, 64)).describe()["kernels"][0]
    assert d["impl"] == "tile_program"
    assert d["row_kernel"] == "interpreter" and "one-row tile" in d["row_kernel_note"]
    wide = CudaExecutable(rowmax_shift_plan(1, 1, 2, 1100)).describe()["kernels"][0]  # 1100 > 1024 columns
    assert wide["row_kernel"] == "interpreter" and "1024" in wide["row_kernel_note"]


def test_fast_row_kernels_build_theirs_for_odd_widths_only():
    # width 128 runs the hand-written kernel: its row program is built only if a launch falls back (unaligned views)
    d = CudaExecutable(workloads.rmsnorm_plan(2, 2, 16, 128)).describe()["kernels"][0]
    assert d["impl"] == "rmsnorm_rows" and d["row_kernel"] == "not built"
    # width 96 is not one the hand-written kernel takes: the fused row program is built at compile time
    d = CudaExecutable(workloads.rmsnorm_plan(2, 2, 16, 96)).describe()["kernels"][0]
    assert d["impl"] == "rmsnorm_rows" and d["row_kernel"] == "compiled"


def test_matmul_with_row_local_epilogue_is_split():
    from _mm_epilogue import mm_epilogue_plan

    if not nvrtc_available():
        pytest.skip("NVRTC not installed")
    d = CudaExecutable(mm_epilogue_plan(1, 256, 256, 256)).describe()["kernels"][0]
    assert d["impl"] == "matmul_tcgen05+row_program", d


def test_kernels_with_contractions_split_into_stages():
    # big tiles: matmul stages (tcgen05 where the operands are f16 params of its shapes, else CUDA cores) and row
    # programs between them; the cycle model is the kernel's own, equal to the oracle's
    import numpy as np
    from _staged import attention_arrays, attention_plan, mlp_arrays, mlp_plan
    from cpu_sim import CpuSim

    for plan, arrays, stages in [
        (attention_plan(1, 1, 1, 256), attention_arrays(np.random.default_rng(0), 1, 1, 1, 256),
         ["matmul 128x256x128 tcgen05", "rows 128", "matmul 128x128x256 cuda_cores", "rows 128"]),
        (mlp_plan(2, 64, 512, 256), mlp_arrays(np.random.default_rng(1), 2, 64, 512, 256),
         ["matmul 64x256x512 cuda_cores", "rows 64", "matmul 64x512x256 cuda_cores", "rows 64"]),
    ]:
        ex = CudaExecutable(plan)
        k = ex.describe()["kernels"][0]
        # the attention tile runs fused on tcgen05 with these stages as its fallback form
        impl = "attention_tcgen05" if plan["name"] == "attention" else "staged_matmul+row_programs"
        assert k["impl"] == impl and k["stages"] == stages and k["scratch_tiles"] == 3
        ex.set_option("dry_run", 1)
        assert ex.run_with_symbols([a.copy() for a in arrays], {}, {}, {}) == CpuSim(plan).run(arrays)
        assert ex.timing()["launches"] == 1  # one batch (its stages launch in order on the GPU)
    # a param the kernel stores to is not re-read by a later stage: its loaded value crosses in scratch
    from _staged import inout_plan

    k = CudaExecutable(inout_plan(2)).describe()["kernels"][0]
    assert k["stages"] == ["rows 128", "matmul 128x128x128 cuda_cores", "rows 128"] and k["scratch_tiles"] == 2


def long_chain_plan(B, R, C, n_ops=45):
    """y = x + (x * 1.5 - ...) over a chain of n_ops element-wise ops (more values than a 32-slot program holds)."""
    kb = KernelBuilder("long_chain")
    x = kb.param("x", "f32", R, C)
    y = kb.param("y", "f32", R, C)
    v = x
    for i in range(n_ops):
        c = kb.op("Constant", [], ("f32", -1, -1), value=1.0 + 0.01 * i)
        v = kb.op(["Mul", "Add", "Sub"][i % 3], [v, c], ("f32", R, C))
    kb.store(y, kb.op("Add", [v, x], ("f32", R, C)))
    body = _pfor("b", B, _task("long_chain", ["b"], [_targ("x", 0, 3, ["b"]), _targ("y", 1, 3, ["b"])]))
    return _plan("long_chain", [("f32", [B, R, C]), ("f32", [B, R, C])], [kb.build()], body, _schedule())


def test_long_op_chains_compile():
    import numpy as np
    from cpu_sim import CpuSim

    plan = long_chain_plan(3, 8, 64)
    ex = CudaExecutable(plan)
    k = ex.describe()["kernels"][0]
    assert k["impl"] == "tile_program" and k["row_kernel"] == "compiled"
    x = np.random.default_rng(0).standard_normal((3, 8, 64)).astype(np.float32)
    ex.set_option("dry_run", 1)
    assert ex.run_with_symbols([x, np.zeros_like(x)], {}, {}, {}) == CpuSim(plan).run([x, np.zeros_like(x)])
