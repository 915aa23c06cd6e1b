"""Drop-in ``target="cuda_sm100a"`` for the reference's unchanged Python API.

The reference has no target registry: ``compile_codegen`` hard-codes
``cpu_sim`` / ``ascend_npu`` (``src/python/pto_codegen.cpp:3352-3434``) and
``Program`` forwards any target string to it (``python/pto_wsp/program.py:437-454``).
``install()`` wraps three ``Program`` methods so that, for the CUDA target only,

* ``_compile_codegen`` converts the workload with the reference's own
  ``workload_to_codegen_ir`` (``python/pto_wsp/ir_bridge.py:112-139``), turns the
  ``ir::Module`` into a plan (``pto_wsp_b200.plan``) and loads it through the
  C-ABI (``ptowsp_cuda_compile``) into a :class:`~pto_wsp_b200.runtime.CudaExecutable`,
  which has the ``CodegenExecutable`` surface (``run_with_symbols``, ``so_path``,
  ``entrypoint``; ``src/python/pto_codegen.cpp:3510-3576``);
* ``_execute_codegen`` runs it on the Program's numpy tensors exactly like the
  CPU-sim path (``program.py:698-733``) but keeps any runtime error;
* ``synchronize`` re-raises that error as the reference's ``ExecutionError``
  (``python/pto_wsp/errors.py:89``) -- the side channel the entry ABI lacks.

Every other target goes to the original methods untouched.
"""

from __future__ import annotations

import threading
import time
from typing import Any, Callable

from .plan import module_to_plan

CUDA_TARGETS = ("cuda_sm100a", "cuda")

_installed = False
_executor_factory: Callable[[dict], Any] | None = None


def _default_factory(plan: dict) -> Any:
    from .runtime import CudaExecutable

    return CudaExecutable(plan)


def install(executor_factory: Callable[[dict], Any] | None = None) -> None:
    """Register the CUDA target on ``pto_wsp.program.Program``.

    ``executor_factory(plan) -> executable`` overrides how a plan is loaded; the
    default is the native runtime.  (Test code passes the CPU oracle here to
    produce golden values from the reference's own example scripts.)
    """
    global _installed, _executor_factory
    _executor_factory = executor_factory
    if _installed:
        return
    from pto_wsp import program as _prog

    Program = _prog.Program
    orig_compile = Program._compile_codegen
    orig_execute = Program._execute_codegen
    orig_sync = Program.synchronize

    def _compile_codegen(self: Any) -> None:
        if str(self.target) not in CUDA_TARGETS:
            return orig_compile(self)
        from pto_wsp.ir_bridge import check_cpp_bindings, workload_to_codegen_ir

        module_name = self.workload._name if getattr(self.workload, "_name", None) else "main"
        check_cpp_bindings()
        build = workload_to_codegen_ir(self.workload, module_name=module_name)
        plan = module_to_plan(build.module)
        factory = _executor_factory or _default_factory
        self._codegen_exec = factory(plan)
        self._can_execute = True
        self._codegen_tensors = build.tensors
        self._cuda_plan = plan

    def _execute_codegen(self: Any) -> None:
        if str(self.target) not in CUDA_TARGETS:
            return orig_execute(self)
        import numpy as np
        from pto_wsp.types import DType

        self.stats.task_count = len(self._compiled_plan.tasks)
        self._cuda_error = None
        zeros = {DType.F32: np.float32, DType.F16: np.float16, DType.I32: np.int32, DType.I64: np.int64,
                 DType.U64: np.uint64, DType.U32: np.uint32}

        def ensure_numpy(t: Any) -> Any:
            if t.data is None:
                if t.dtype not in zeros:
                    raise ValueError(f"Unsupported dtype for codegen runtime: {t.dtype}")
                t.data = np.zeros(t.shape, dtype=zeros[t.dtype])
            if not isinstance(t.data, np.ndarray):
                raise TypeError(f"Tensor.data must be a numpy.ndarray for codegen runtime (got {type(t.data)})")
            return t.data

        def run() -> None:
            try:
                arrays = [ensure_numpy(t) for t in self._codegen_tensors]
                axis_sizes = {str(k): int(v) for k, v in self._axis_sizes.items()}
                t0 = time.perf_counter()
                cycles = self._codegen_exec.run_with_symbols(
                    arrays, axis_sizes, dict(self._symbols_u64), dict(self._symbols_ptr))
                self.stats.total_cycles = int(cycles)
                self._cuda_wall_ms = (time.perf_counter() - t0) * 1000.0
            except BaseException as e:  # noqa: BLE001 - surfaced by synchronize()
                self._cuda_error = e
            finally:
                self._complete.set()

        self._codegen_thread = threading.Thread(target=run, daemon=True)
        self._codegen_thread.start()

    def synchronize(self: Any) -> None:
        orig_sync(self)
        err = getattr(self, "_cuda_error", None) if str(self.target) in CUDA_TARGETS else None
        if err is not None:
            self._cuda_error = None
            from pto_wsp.errors import ExecutionError

            raise ExecutionError(f"cuda_sm100a execution failed: {err}") from err

    Program._compile_codegen = _compile_codegen
    Program._execute_codegen = _execute_codegen
    Program.synchronize = synchronize
    _installed = True
