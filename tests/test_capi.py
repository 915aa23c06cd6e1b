"""The C-ABI library loads, exports every declared symbol, and fails loudly without a GPU (CPU)."""

import re
from pathlib import Path

import pytest

from golden_cases import load_cases
from pto_wsp_b200 import runtime, workloads
from pto_wsp_b200.plan import dumps

HDR = Path(__file__).resolve().parents[1] / "include" / "ptowsp_cuda.h"


def declared_functions() -> list[str]:
    text = HDR.read_text()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(ptowsp_cuda_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "ptowsp_cuda_compile" in names and "ptowsp_cuda_main" in names and "ptowsp_cuda_run_task" in names


def test_library_exports_every_declared_symbol():
    lib = runtime.load_library()
    for name in declared_functions():
        assert hasattr(lib, name), name


@pytest.mark.parametrize("idx", range(len(load_cases())))
def test_compile_fixture_plans(idx):
    case = load_cases()[idx]
    ex = runtime.CudaExecutable(case["plan"])
    d = ex.describe()
    assert len(d["kernels"]) == len(case["plan"]["kernels"])


@pytest.mark.parametrize("plan,impls", [
    (workloads.rmsnorm_plan(4, 64), ["rmsnorm_rows"]),
    (workloads.softmax_plan(32, 2048), ["softmax_rows"]),
    (workloads.bgemm_plan(2, 256, 256, 512), ["matmul_tcgen05"]),
    (workloads.bgemm_plan(2, 256, 256, 512, accumulate=True), ["matmul_tcgen05_acc"]),
    (workloads.decode_plan(4, 8, 4, 128, 100, 64), ["paged_decode_gqa"]),
    (workloads.indexer_plan(2, 8, 64, 128, 1024, 64), ["lightning_indexer_score", "topk_select"]),
])
def test_config_kernels_match_hand_written_impls(plan, impls):
    d = runtime.CudaExecutable(plan).describe()
    assert [k["impl"] for k in d["kernels"]] == impls


def test_cpu_body_kernels_are_rejected():
    plan = workloads.rmsnorm_plan(1, 1)
    plan["kernels"][0]["attrs"] = {"cpp_src": "  // CPU body\n"}
    with pytest.raises(runtime.PtoWspCudaError) as e:
        runtime.CudaExecutable(plan)
    assert e.value.code == 2 and "CPU C++ body" in str(e.value)


def test_malformed_plans_are_rejected():
    with pytest.raises(runtime.PtoWspCudaError) as e:
        runtime.CudaExecutable({"format": "ptowsp-plan/1", "name": "x", "tensors": [], "kernels": [],
                                "body": {"kind": "task", "kernel": "missing", "axis_args": [], "scalar_args": [],
                                         "tensor_args": []}})
    assert e.value.code == 1 and "Missing kernel def" in str(e.value)
    lib = runtime.load_library()
    import ctypes as C

    h = C.c_void_p()
    bad = b"{not json"
    assert lib.ptowsp_cuda_compile(bad, len(bad), 0, C.byref(h)) == 1


def test_run_without_gpu_fails_loudly():
    if runtime.device_count() > 0:
        pytest.skip("a GPU is present")
    import numpy as np

    ex = runtime.CudaExecutable(workloads.rmsnorm_plan(1, 2))
    x = np.ones((1, 2, 16, 128), np.float32)
    y = np.zeros_like(x)
    with pytest.raises(runtime.PtoWspCudaError) as e:
        ex.run_with_symbols([x, y], {}, {}, {})
    assert e.value.code == 3
    assert not y.any()  # no CPU fallback wrote anything


@pytest.mark.parametrize("idx", range(len(load_cases())), ids=[c["name"] for c in load_cases()])
def test_native_cycle_model_matches_oracle_dry_run(idx):
    """The C++ walk + cycle model gives the CPU-sim makespan for every reference case (host only)."""
    from golden_cases import materialize

    case = load_cases()[idx]
    roots, arrays, axis, syms, sptr = materialize(case, idx)
    ex = runtime.CudaExecutable(case["plan"])
    ex.set_option("dry_run", 1)
    assert ex.run_with_symbols(arrays, axis, syms, sptr) == case["cycles"]


def test_dry_run_waves_and_staging():
    import numpy as np

    ex = runtime.CudaExecutable(workloads.softmax_plan(4, 16))
    ex.set_option("dry_run", 1)
    x = np.zeros((4, 16, 32, 256), np.float32)
    y = np.zeros_like(x)
    c = ex.run_with_symbols([x, y], {}, {}, {})
    t = ex.timing()
    assert t["tasks"] == 64 and t["waves"] == 1 and t["launches"] == 1
    assert t["h2d_bytes"] == x.nbytes and t["d2h_bytes"] == y.nbytes  # write-only output is not staged in
    assert c > 0


def test_dry_run_intermediate_written_before_read_is_not_staged_in():
    import numpy as np

    # the indexer's scores: written in full by the scoring wave, read only by the top-k wave after it
    plan, arrays = workloads.indexer_inputs(np.random.default_rng(0), 2, 4096, 256)
    ex = runtime.CudaExecutable(plan)
    ex.set_option("dry_run", 1)
    ex.run_with_symbols(arrays, {}, {}, {})
    t = ex.timing()
    assert t["waves"] == 2
    assert t["h2d_bytes"] == sum(a.nbytes for a in arrays[:3])  # q, k, w
    assert t["d2h_bytes"] == arrays[3].nbytes + arrays[4].nbytes  # scores and indices come back
    # accumulate form: C is read by the task that writes it, so it is staged in
    plan = workloads.bgemm_plan(1, 256, 256, 128, accumulate=True)
    ex = runtime.CudaExecutable(plan)
    ex.set_option("dry_run", 1)
    a = np.zeros((1, 256, 128), np.float16)
    b = np.zeros((1, 128, 256), np.float16)
    c = np.zeros((1, 256, 256), np.float32)
    ex.run_with_symbols(list(workloads.bgemm_views(a, b, c)), {}, {}, {})
    assert ex.timing()["h2d_bytes"] == a.nbytes + b.nbytes + c.nbytes


def test_dry_run_inout_chain_waves():
    import numpy as np

    # bgemm k-tile accumulation form: C[b][i][j] += A . B over P.seq(k) -> one wave per k step
    from golden_cases import case_index, materialize

    cases = load_cases()
    idx = case_index(cases, "example:bgemm#0")
    roots, arrays, axis, syms, sptr = materialize(cases[idx], idx)
    ex = runtime.CudaExecutable(cases[idx]["plan"])
    ex.set_option("dry_run", 1)
    ex.run_with_symbols(arrays, axis, syms, sptr)
    t = ex.timing()
    assert t["tasks"] == 64 and t["waves"] == 4


@pytest.mark.parametrize("name", ["rmsnorm", "softmax", "bgemm", "decode", "indexer", "topk"])
def test_native_cycles_match_oracle_for_config_plans(name):
    """Dry-run makespan of the native runtime == the oracle's, for every config workload form."""
    import numpy as np
    from cpu_sim import CpuSim

    rng = np.random.default_rng(0)
    axis = {}
    if name == "rmsnorm":
        plan = workloads.rmsnorm_plan(2, 3)
        arrays = [np.zeros((2, 3, 16, 128), np.float32) for _ in range(2)]
    elif name == "softmax":
        plan = workloads.softmax_plan(2, 3)
        arrays = [np.zeros((2, 3, 32, 256), np.float32) for _ in range(2)]
    elif name == "bgemm":
        plan = workloads.bgemm_plan(1, 256, 256, 128)
        a, b, c = np.zeros((1, 256, 128), np.float16), np.zeros((1, 128, 256), np.float16), np.zeros((1, 256, 256), np.float32)
        arrays = list(workloads.bgemm_views(a, b, c))
    elif name == "decode":
        plan, arrays = workloads.decode_inputs(rng, 3, lengths=[5, 40, 0])
        axis = {"b": 3}
    elif name == "indexer":
        plan, arrays = workloads.indexer_inputs(rng, 1, 256, 16)
    else:
        plan = workloads.topk_plan(3, 256, 16)
        arrays = [np.zeros((3, 1, 256), np.float32), np.zeros((3, 1, 16), np.int32)]
    want = CpuSim(plan).run([x.copy() for x in arrays], axis_sizes=axis, execute=False)
    ex = runtime.CudaExecutable(plan)
    ex.set_option("dry_run", 1)
    assert ex.run_with_symbols(arrays, axis, {}, {}) == want


def test_tensor_driven_tiers_are_device_selected_and_cacheable():
    """`P.when` tiers over a slot loaded from a tensor, with leaves that differ only in scalars: the walk no longer
    reads the data (the plan is cacheable) and its makespan still equals the oracle's."""
    import numpy as np
    from _dev_select import tiered_scale_plan
    from cpu_sim import CpuSim

    from pto_wsp_b200.runtime import CudaExecutable

    plan = tiered_scale_plan(3, 5)
    ex = CudaExecutable(plan)
    assert ex.describe()["cacheable"]
    rng = np.random.default_rng(0)
    sel = rng.integers(-20, 200, (3, 5, 1, 1)).astype(np.int32)
    x = rng.standard_normal((3, 5, 8, 64)).astype(np.float32)
    out = np.zeros_like(x)
    want = CpuSim(plan).run([sel, x, out.copy()])
    ex.set_option("dry_run", 1)
    assert ex.run_with_symbols([sel, x, out], {}, {}, {}) == want


def _two_wave_plan(B, T, R, C, swap=False, write_back_x=False):
    """Wave 0: M[b, t] = X[b, t] * 2; wave 1: Y[b, t] = M[b, t] + 1 (loops t-outer when `swap`; when
    `write_back_x` the second kernel writes X instead of Y).  Tensors: 0 = X, 1 = M, 2 = Y, all [B, T, R, C] f32."""
    from pto_wsp_b200.workloads import KernelBuilder, _pfor, _plan, _schedule, _targ, _task

    k1 = KernelBuilder("scale")
    x = k1.param("x", "f32", R, C)
    m = k1.param("m", "f32", R, C)
    two = k1.op("Constant", [], ("f32", -1, -1), value=2.0)
    k1.store(m, k1.op("Mul", [x, two], ("f32", R, C)))
    k2 = KernelBuilder("shift")
    m2 = k2.param("m", "f32", R, C)
    y = k2.param("y", "f32", R, C)
    one = k2.op("Constant", [], ("f32", -1, -1), value=1.0)
    k2.store(y, k2.op("Add", [m2, one], ("f32", R, C)))
    n1 = _pfor("b", B, _pfor("t", T, _task("scale", ["b", "t"], [_targ("x", 0, 4, ["b", "t"]),
                                                                 _targ("m", 1, 4, ["b", "t"])])))
    task2 = _task("shift", ["b2", "t2"], [_targ("m", 1, 4, ["b2", "t2"]),
                                          _targ("y", 0 if write_back_x else 2, 4, ["b2", "t2"])])
    n2 = _pfor("t2", T, _pfor("b2", B, task2)) if swap else _pfor("b2", B, _pfor("t2", T, task2))
    shape = [B, T, R, C]
    return _plan("two_wave", [("f32", shape)] * 3, [k1.build(), k2.build()], {"kind": "combine", "children": [n1, n2]},
                 _schedule())


def test_dry_run_reports_overlapped_chunks():
    import numpy as np

    # one batch, 64 MiB in + 64 MiB out: 32 chunks (4 MiB of host traffic each at least, at most 32)
    ex = runtime.CudaExecutable(workloads.softmax_plan(2, 1024))
    ex.set_option("dry_run", 1)
    x = np.zeros((2, 1024, 32, 256), np.float32)
    ex.run_with_symbols([x, np.zeros_like(x)], {}, {}, {})
    assert ex.timing()["chunks"] == 32
    ex.set_option("pipeline_chunks", 8)
    ex.run_with_symbols([x, np.zeros_like(x)], {}, {}, {})
    assert ex.timing()["chunks"] == 8
    ex.set_option("pipeline_chunks", 1)
    ex.run_with_symbols([x, np.zeros_like(x)], {}, {}, {})
    assert ex.timing()["chunks"] == 0
    # small host buffers: not worth the extra streams
    ex = runtime.CudaExecutable(workloads.softmax_plan(2, 16))
    ex.set_option("dry_run", 1)
    x = np.zeros((2, 16, 32, 256), np.float32)
    ex.run_with_symbols([x, np.zeros_like(x)], {}, {}, {})
    assert ex.timing()["chunks"] == 0


@pytest.mark.parametrize("swap,write_back_x,chunks", [(False, False, 16), (True, False, 0), (False, True, 0)])
def test_dry_run_chain_pipelining_rules(swap, write_back_x, chunks):
    # two waves chunk by chunk when chunk c of the reader reads inside what chunk c of the writer wrote (same loop
    # order); not when the reader walks the intermediate in another order, nor when a wave writes what an
    # earlier wave read
    import numpy as np

    B, T, R, C = 8, 128, 32, 256  # 32 MiB per tensor
    ex = runtime.CudaExecutable(_two_wave_plan(B, T, R, C, swap, write_back_x))
    ex.set_option("dry_run", 1)
    ex.set_option("pipeline_chunks", 16)
    arrays = [np.zeros((B, T, R, C), np.float32) for _ in range(3)]
    ex.run_with_symbols(arrays, {}, {}, {})
    t = ex.timing()
    assert t["waves"] == 2 and t["chunks"] == chunks
    if not write_back_x:  # M is written in full before it is read: never staged in
        assert t["h2d_bytes"] == arrays[0].nbytes


def test_tiles_larger_than_their_views_are_ordered():
    """The reference softmax example indexes its tiles one dimension too shallow, so each [8, 64] tile reaches
    8 rows from a [4, 64] view into the next views.  The CPU-sim runs tasks in program order; here every task
    that writes such a tensor gets its own wave (whole-tensor hazard key): 4 max-update steps (P.seq over v) +
    16 exp/accumulate + 16 rescale tasks."""
    from golden_cases import case_index, load_cases, materialize

    cases = load_cases()
    idx = case_index(cases, "example:softmax#0")
    roots, arrays, axis, syms, sptr = materialize(cases[idx], idx)
    ex = runtime.CudaExecutable(cases[idx]["plan"])
    ex.set_option("dry_run", 1)
    assert ex.run_with_symbols(arrays, axis, syms, sptr) == cases[idx]["cycles"]
    assert ex.timing()["waves"] == 36 and ex.timing()["tasks"] == 48
