"""Generate golden fixtures from the reference's own scripts (build container only).

Runs, unchanged, the reference's example drivers (``examples/*/*_example.py``)
and its codegen execution tests (``tests/test_codegen_*.py``) with the CUDA
target redirected through ``pto_wsp_b200.frontend``: the reference frontend
builds each workload and ``ir::Module``, the plan is recorded, and the CPU
oracle (``oracle/cpu_sim.py``) executes it.  The reference scripts then apply
their own checks -- numpy goldens, exact ``atol=0`` outputs, exact cycle counts
-- to the oracle's results, which pins the oracle.

Every module is also compiled by the reference's own codegen into its CPU-sim
artifact (``workload_main.cpp`` + ``kernel_*.cpp``, built by oracle/Makefile's
``ref`` module with the clean-room pto-isa stand-in ``oracle/ptoisa``) and run
through the reference's own ``CodegenExecutable`` on a copy of the same
inputs: its cycle count must equal the oracle's, and its output buffers are
saved beside the oracle's (``c<i>_art<j>``) so that the CPU tests hold the two
against each other.  Every run is saved as a case: plan, input buffers (with
the exact numpy view layout), axis sizes, symbols, the oracle's and the
artifact's output buffers and the cycle count.

    PTOWSP_REFERENCE=<reference checkout> python tests/golden/make_golden.py

Kernels with CPU C++ bodies (``cpp_src``) are skipped: the CUDA target rejects them.  That includes
``@ptoisa_kernel`` kernels (``tests/test_ptoisa_kernel_jit.py``), whose traced PTO-ISA calls reach the plan
only as generated C++ source.
"""

from __future__ import annotations

import importlib
import io
import json
import os
import runpy
import sys
from contextlib import redirect_stdout
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "oracle")]
from refpath import reference_root  # noqa: E402

REF = reference_root()
if REF is None:
    raise SystemExit("reference checkout not found: set PTOWSP_REFERENCE")
sys.path[:0] = [str(ROOT / "oracle" / "_ref"), str(REF / "python")]

from cpu_sim import CpuSim  # noqa: E402

from pto_wsp_b200 import frontend  # noqa: E402

CASES: list[dict] = []
ARRAYS: dict[str, np.ndarray] = {}
CURRENT = {"name": "?", "tol": (0.0, 0.0)}
LAST_MODULE: dict = {}  # the ir::Module of the workload being compiled (for its CPU-sim artifact)


def _root(a: np.ndarray) -> np.ndarray:
    r = a
    while isinstance(r.base, np.ndarray):
        r = r.base
    return r


def _layout(arrays: list[np.ndarray], prefix: str) -> tuple[list[dict], list[np.ndarray]]:
    owners: list[np.ndarray] = []  # the arrays owning the memory (identity: views of one buffer share it)
    roots: list[np.ndarray] = []   # the same memory as saved: C-contiguous, or a dense buffer in another axis
    descs = []                     # order (``transpose(...).astype(...)``) flattened in memory order
    for a in arrays:
        r = _root(a)
        ri = next((i for i, x in enumerate(owners) if x is r), None)
        if ri is None:
            owners.append(r)
            flat = r if r.flags.c_contiguous else r.ravel(order="K")
            assert np.may_share_memory(flat, r), "tensor memory is not one dense buffer"
            roots.append(flat)
            ri = len(roots) - 1
        r = roots[ri]
        off = a.__array_interface__["data"][0] - r.__array_interface__["data"][0]
        descs.append({"root": ri, "dtype": a.dtype.str, "shape": list(a.shape), "strides": list(a.strides),
                      "offset": int(off)})
    return descs, roots


def _artifact(module):
    """The reference CPU-sim artifact of `module`, loaded through the reference's own CodegenExecutable."""
    from pto_wsp.ir_bridge import cpp

    opts = cpp.CompileOptions()
    opts.target = "cpu_sim"
    res = cpp.compile_codegen(module, opts)
    return cpp.CodegenExecutable(str(res["so_path"]), str(res["entrypoint"]))


def _views_on(descs, roots):
    return [np.ndarray(shape=tuple(d["shape"]), dtype=np.dtype(d["dtype"]), buffer=roots[d["root"]],
                       offset=d["offset"], strides=tuple(d["strides"])) for d in descs]


class RecordingExecutable:
    so_path = "<oracle>"

    def __init__(self, plan: dict):
        self.plan = plan
        self.entrypoint = f"{plan.get('name', 'main')}_main"
        self.sim = CpuSim(plan)
        self.art = _artifact(LAST_MODULE["module"])

    def run_with_symbols(self, arrays, axis_sizes, symbols_u64, symbols_ptr):
        arrays = list(arrays)
        sp_keys = sorted(symbols_ptr)
        sp_arrays = [np.asarray(symbols_ptr[k]) for k in sp_keys]
        descs, roots = _layout(arrays + sp_arrays, "")
        idx = len(CASES)
        name = f"{CURRENT['name']}#{sum(1 for c in CASES if c['name'].startswith(CURRENT['name'] + '#'))}"
        for i, r in enumerate(roots):
            ARRAYS[f"c{idx}_in{i}"] = np.frombuffer(r.tobytes(), dtype=np.uint8).copy()
        # the reference's own artifact first, on a copy laid out exactly like the caller's buffers
        art_roots = [r.copy() for r in roots]
        art_views = _views_on(descs, art_roots)
        art_cycles = int(self.art.run_with_symbols(
            art_views[: len(arrays)], dict(axis_sizes), dict(symbols_u64),
            {k: v for k, v in zip(sp_keys, art_views[len(arrays):])}))
        cycles = self.sim.run(arrays, axis_sizes, symbols_u64, symbols_ptr)
        if art_cycles != int(cycles):
            raise SystemExit(f"{name}: CPU-sim artifact cycles {art_cycles} != oracle {cycles}")
        for i, r in enumerate(roots):
            ARRAYS[f"c{idx}_out{i}"] = np.frombuffer(r.tobytes(), dtype=np.uint8).copy()
            ARRAYS[f"c{idx}_art{i}"] = np.frombuffer(art_roots[i].tobytes(), dtype=np.uint8).copy()
            ARRAYS[f"c{idx}_dtype{i}"] = np.frombuffer(r.dtype.str.encode(), dtype=np.uint8).copy()
        CASES.append({
            "name": name, "plan": self.plan, "arrays": descs[: len(arrays)], "symbols_ptr": [
                {"id": str(k), **d} for k, d in zip(sp_keys, descs[len(arrays):])],
            "roots": [{"dtype": r.dtype.str, "shape": list(r.shape)} for r in roots],
            "axis_sizes": {str(k): int(v) for k, v in axis_sizes.items()},
            "symbols_u64": {str(k): int(v) for k, v in symbols_u64.items()},
            "cycles": int(cycles), "rtol": CURRENT["tol"][0], "atol": CURRENT["tol"][1],
        })
        return cycles

    def run(self, arrays, axis_sizes):
        return self.run_with_symbols(arrays, axis_sizes, {}, {})


def _redirect_cpu_sim():
    W = importlib.import_module("pto_wsp.workload")
    orig = W.Workload.compile

    def comp(self, target="cpu_sim", **kw):
        return orig(self, target="cuda_sm100a" if target == "cpu_sim" else target, **kw)

    W.Workload.compile = comp
    B = importlib.import_module("pto_wsp.ir_bridge")
    orig_w2ir = B.workload_to_codegen_ir

    def w2ir(*a, **kw):
        build = orig_w2ir(*a, **kw)
        LAST_MODULE["module"] = build.module
        return build

    B.workload_to_codegen_ir = w2ir


EXAMPLES = [
    ("attention", (1e-2, 1e-2)),
    ("llama", (1e-5, 1e-6)),
    ("deepseek_v3", (1e-5, 1e-6)),
    ("validated_matmul", (1e-5, 1e-6)),
    ("tensor_data", (1e-5, 1e-6)),
    ("e2e_rmsnorm", (1e-5, 1e-6)),
    ("softmax", (1e-2, 1e-2)),
    ("bgemm", (1e-2, 1e-2)),
    ("flashinfer_decode", (1e-5, 1e-6)),
    ("deepseek_lightning_indexer", (0.0, 0.0)),
    ("csp_pipeline", (1e-6, 1e-6)),
]

REF_TESTS = [
    ("test_e2e.py", (0.0, 0.0)),
    ("test_codegen_execute_basic.py", (0.0, 0.0)),
    ("test_codegen_dynamic_axes.py", (0.0, 0.0)),
    ("test_codegen_schedule_dispatch_window.py", (0.0, 0.0)),
    ("test_codegen_dynamic_symbols.py", (0.0, 0.0)),
    ("test_codegen_ragged_axis.py", (0.0, 0.0)),
    ("test_codegen_select_sparse.py", (0.0, 0.0)),
    ("test_codegen_cond.py", (0.0, 0.0)),
    ("test_codegen_scalar_expr_eval.py", (0.0, 0.0)),
    ("test_kernel_tracing_codegen.py", (1e-5, 1e-6)),
    ("test_codegen_cspt_pipeline.py", (0.0, 0.0)),
]


def main() -> None:
    frontend.install(RecordingExecutable)
    _redirect_cpu_sim()
    ok = True
    for ex, tol in EXAMPLES:
        d = REF / "examples" / ex
        sys.path[:0] = [str(d), str(REF / "examples" / "_harness")]
        for m in ("pto_wsp_impl", "golden", "harness"):
            sys.modules.pop(m, None)
        CURRENT["name"], CURRENT["tol"] = f"example:{ex}", tol
        if ex == "deepseek_lightning_indexer":
            os.environ["PTO_WSP_DEEPSEEK_LIGHTNING_INDEXER_IMPL"] = "pto"
        buf = io.StringIO()
        with redirect_stdout(buf):
            if ex == "csp_pipeline":
                # its script defines a second, stale main() after the __main__ guard: run it as a script
                try:
                    runpy.run_path(str(d / f"{ex}_example.py"), run_name="__main__")
                    res = True
                except SystemExit as e:
                    res = e.code in (0, None)
            else:
                res = runpy.run_path(str(d / f"{ex}_example.py"), run_name="ptowsp_example")["main"]()
        print(f"{ex}: {'PASS' if res else 'FAIL'}  {buf.getvalue().strip().splitlines()[-1]}")
        ok &= bool(res)
        sys.path[:2] = []
    import pytest

    for tf, tol in REF_TESTS:
        CURRENT["name"], CURRENT["tol"] = f"reftest:{tf}", tol
        rc = pytest.main(["-q", "-p", "no:cacheprovider", "--rootdir", "/tmp", str(REF / "tests" / tf)])
        print(f"{tf}: {'PASS' if rc == 0 else 'FAIL'}")
        ok &= rc == 0
    if not ok:
        raise SystemExit("reference checks failed against the oracle; fixtures not written")
    (HERE / "ref_cases.json").write_text(json.dumps(CASES, sort_keys=True, indent=1))
    np.savez_compressed(HERE / "ref_cases.npz", **ARRAYS)
    print(f"wrote {len(CASES)} cases")


if __name__ == "__main__":
    main()
