"""ctypes binding of ``libptowsp_cuda.so`` (C ABI in ``include/ptowsp_cuda.h``).

:class:`CudaExecutable` has the surface of the reference's ``CodegenExecutable``
(``src/python/pto_codegen.cpp:3510-3576``): ``run_with_symbols(arrays,
axis_sizes, symbols_u64, symbols_ptr)`` builds the reference ``RuntimeContext``
(``include/pto/wsp/codegen/abi/workload_abi.hpp:17-41``) -- tensor pointers,
element strides, axis sizes by loop-variable name, FNV-1a symbol ids and 256
u64 slots (``pto_codegen.cpp:3453-3505``) -- and calls the native entry point.
Arrays may be numpy arrays (host memory, staged to HBM and back by the
runtime) or CUDA tensors / ``__cuda_array_interface__`` objects (used in
place).  There is no CPU fallback: without the native library or a GPU the
calls raise.
"""

from __future__ import annotations

import ctypes as C
import json
import os
from pathlib import Path
from typing import Any

from .plan import dumps

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libptowsp_cuda.so"

PTOWSP_OK = 0

_AXIS_FN = C.CFUNCTYPE(C.c_int64, C.c_void_p, C.c_char_p)
_SYMU_FN = C.CFUNCTYPE(C.c_uint64, C.c_void_p, C.c_uint64)
_SYMP_FN = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.c_uint64)
_SLOTG_FN = C.CFUNCTYPE(C.c_uint64, C.c_void_p, C.c_uint32)
_SLOTS_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_uint32, C.c_uint64)
_TPTR_FN = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.c_uint32)
_TSTR_FN = C.CFUNCTYPE(C.c_uint64, C.c_void_p, C.c_uint32, C.c_uint32)
_KERN_FN = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.c_uint32)


class RuntimeContext(C.Structure):
    _fields_ = [
        ("get_axis_size", _AXIS_FN),
        ("get_symbol_u64", _SYMU_FN),
        ("get_symbol_ptr", _SYMP_FN),
        ("get_slot_u64", _SLOTG_FN),
        ("set_slot_u64", _SLOTS_FN),
        ("get_tensor_ptr", _TPTR_FN),
        ("get_tensor_stride", _TSTR_FN),
        ("get_kernel", _KERN_FN),
        ("ctx", C.c_void_p),
    ]


class KernelTaskDesc(C.Structure):
    _fields_ = [
        ("args", C.POINTER(C.c_uint64)),
        ("num_args", C.c_uint32),
        ("num_axis_args", C.c_uint32),
        ("tensor_ptrs", C.POINTER(C.c_void_p)),
        ("tensor_strides", C.POINTER(C.c_uint64)),
        ("num_tensors", C.c_uint32),
        ("kernel_id", C.c_uint32),
        ("task_id", C.c_uint32),
    ]


class Timing(C.Structure):
    _fields_ = [
        ("gpu_ms", C.c_double),
        ("total_ms", C.c_double),
        ("launches", C.c_uint64),
        ("tasks", C.c_uint64),
        ("waves", C.c_uint64),
        ("h2d_bytes", C.c_uint64),
        ("d2h_bytes", C.c_uint64),
        ("slot_syncs", C.c_uint64),
        ("chunks", C.c_uint64),
        ("walks", C.c_uint64),
        ("expansions", C.c_uint64),
    ]


_lib: C.CDLL | None = None


def library_path() -> Path:
    return Path(os.environ.get("PTOWSP_CUDA_LIB", str(LIB_PATH)))


def load_library() -> C.CDLL:
    """Load the native library; raises if it was not built (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.exists():
        raise RuntimeError(f"native library missing: {path} (run `python -m pto_wsp_b200.build`)")
    lib = C.CDLL(str(path))
    lib.ptowsp_cuda_compile.argtypes = [C.c_char_p, C.c_size_t, C.c_int, C.POINTER(C.c_void_p)]
    lib.ptowsp_cuda_compile.restype = C.c_int
    lib.ptowsp_cuda_main.argtypes = [C.c_void_p, C.POINTER(RuntimeContext), C.c_void_p]
    lib.ptowsp_cuda_main.restype = C.c_uint64
    lib.ptowsp_cuda_run_task.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(KernelTaskDesc)]
    lib.ptowsp_cuda_run_task.restype = C.c_uint64
    lib.ptowsp_cuda_status.argtypes = [C.c_void_p]
    lib.ptowsp_cuda_status.restype = C.c_int
    lib.ptowsp_cuda_last_error.argtypes = []
    lib.ptowsp_cuda_last_error.restype = C.c_char_p
    lib.ptowsp_cuda_set_stream.argtypes = [C.c_void_p, C.c_void_p]
    lib.ptowsp_cuda_set_stream.restype = C.c_int
    lib.ptowsp_cuda_set_option.argtypes = [C.c_void_p, C.c_char_p, C.c_int64]
    lib.ptowsp_cuda_set_option.restype = C.c_int
    lib.ptowsp_cuda_last_timing.argtypes = [C.c_void_p, C.POINTER(Timing)]
    lib.ptowsp_cuda_last_timing.restype = C.c_int
    lib.ptowsp_cuda_kernel_times.argtypes = [C.c_void_p]
    lib.ptowsp_cuda_kernel_times.restype = C.c_char_p
    lib.ptowsp_cuda_describe.argtypes = [C.c_void_p]
    lib.ptowsp_cuda_describe.restype = C.c_char_p
    lib.ptowsp_cuda_destroy.argtypes = [C.c_void_p]
    lib.ptowsp_cuda_destroy.restype = None
    lib.ptowsp_cuda_device_count.argtypes = []
    lib.ptowsp_cuda_device_count.restype = C.c_int
    _lib = lib
    return lib


class PtoWspCudaError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[ptowsp_cuda status {code}] {message}")
        self.code = code


def _last_error() -> str:
    m = load_library().ptowsp_cuda_last_error()
    return m.decode() if m else ""


def _array_info(a: Any) -> tuple[int, list[int]]:
    """(data pointer, element strides) of a numpy array / CUDA tensor."""
    if hasattr(a, "data_ptr") and hasattr(a, "stride"):  # torch.Tensor
        return int(a.data_ptr()), [int(s) for s in a.stride()]
    if hasattr(a, "__cuda_array_interface__"):
        cai = a.__cuda_array_interface__
        import numpy as np

        item = np.dtype(cai["typestr"]).itemsize
        shape = cai["shape"]
        strides = cai.get("strides")
        if strides is None:
            strides, acc = [], 1
            for d in reversed(shape):
                strides.insert(0, acc)
                acc *= d
        else:
            strides = [s // item for s in strides]
        return int(cai["data"][0]), list(strides)
    import numpy as np

    if not isinstance(a, np.ndarray):
        raise TypeError(f"tensor data must be a numpy array or CUDA tensor (got {type(a)})")
    return int(a.ctypes.data), [s // a.itemsize for s in a.strides]


def device_count() -> int:
    return int(load_library().ptowsp_cuda_device_count())


class CudaExecutable:
    """A compiled plan; drop-in for the reference ``CodegenExecutable``."""

    def __init__(self, plan: dict, device: int = 0):
        lib = load_library()
        self.plan = plan
        self.device = device
        self.so_path = str(library_path())
        self.entrypoint = f"{plan.get('name', 'main')}_main"
        text = dumps(plan).encode()
        h = C.c_void_p()
        rc = lib.ptowsp_cuda_compile(text, len(text), int(device), C.byref(h))
        if rc != PTOWSP_OK:
            raise PtoWspCudaError(rc, _last_error())
        self._h = h
        self._lib = lib

    def __del__(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self._lib.ptowsp_cuda_destroy(h)
            self._h = None

    # -- reference surface --------------------------------------------------
    def run(self, arrays, axis_sizes) -> int:
        return self.run_with_symbols(arrays, axis_sizes, {}, {})

    def _context(self) -> RuntimeContext:
        """The RuntimeContext of this executable: its callbacks are made once and read ``self._call``, the
        current call's tensors, axis sizes, symbols and slots (the reference builds the same struct per run,
        ``pto_codegen.cpp:3453-3505``)."""
        if getattr(self, "_ctx", None) is None:
            st = self._call = {"infos": [], "axis": {}, "syms": {}, "sptr": {}, "slots": [0] * 256}

            def get_axis_size(_ctx, name):
                return st["axis"].get(name, 0)

            def get_symbol_u64(_ctx, sid):
                return st["syms"].get(sid, 0)

            def get_symbol_ptr(_ctx, sid):
                return st["sptr"].get(sid, None)

            def get_slot_u64(_ctx, i):
                return st["slots"][i] if i < 256 else 0

            def set_slot_u64(_ctx, i, v):
                if i < 256:
                    st["slots"][i] = v

            def get_tensor_ptr(_ctx, tid):
                infos = st["infos"]
                return infos[tid][0] if tid < len(infos) else None

            def get_tensor_stride(_ctx, tid, dim):
                infos = st["infos"]
                if tid >= len(infos) or dim >= len(infos[tid][1]):
                    return 0
                return infos[tid][1][dim] & 0xFFFFFFFFFFFFFFFF

            def get_kernel(_ctx, kid):
                return None

            self._cbs = (_AXIS_FN(get_axis_size), _SYMU_FN(get_symbol_u64), _SYMP_FN(get_symbol_ptr),
                         _SLOTG_FN(get_slot_u64), _SLOTS_FN(set_slot_u64), _TPTR_FN(get_tensor_ptr),
                         _TSTR_FN(get_tensor_stride), _KERN_FN(get_kernel))
            self._ctx = RuntimeContext(*self._cbs, None)
        return self._ctx

    def run_with_symbols(self, arrays, axis_sizes, symbols_u64, symbols_ptr) -> int:
        ctx = self._context()
        st = self._call
        st["infos"] = [_array_info(a) for a in arrays]
        st["axis"] = {str(k).encode(): int(v) for k, v in (axis_sizes or {}).items()}
        st["syms"] = {int(k) & 0xFFFFFFFFFFFFFFFF: int(v) & 0xFFFFFFFFFFFFFFFF for k, v in (symbols_u64 or {}).items()}
        st["sptr"] = {int(k) & 0xFFFFFFFFFFFFFFFF: _array_info(v)[0] for k, v in (symbols_ptr or {}).items()}
        st["slots"] = [0] * 256  # slots start at zero every run
        keep = (arrays, symbols_ptr)  # alive for the call
        try:
            cycles = self._lib.ptowsp_cuda_main(self._h, C.byref(ctx), None)
        finally:
            st["infos"], st["sptr"] = [], {}
            del keep
        rc = self._lib.ptowsp_cuda_status(self._h)
        if rc != PTOWSP_OK:
            raise PtoWspCudaError(rc, _last_error())
        return int(cycles)

    # -- extras -------------------------------------------------------------
    def run_task(self, kernel: str, tensors: list[Any], axis_args: list[int] = (), scalar_args: list[int] = ()) -> int:
        """Run one task of `kernel` on device tensors (the per-kernel reference ABI)."""
        kd = next(k for k in self.plan["kernels"] if k["name"] == kernel)
        vals = {v[0]: v for v in kd["values"]}
        tparams = [p for p in kd["params"] if vals[p["id"]][2] >= 0]
        tail = []
        for p in tparams:
            tail += [vals[p["id"]][2], vals[p["id"]][3]]
        args = list(axis_args) + tail + list(scalar_args)
        arr_args = (C.c_uint64 * max(len(args), 1))(*[int(a) & 0xFFFFFFFFFFFFFFFF for a in args])
        ptrs, strides = [], []
        for t in tensors:
            ptr, st = _array_info(t)
            ptrs.append(ptr)
            strides += [st[-2] if len(st) >= 2 else 0, st[-1] if st else 1]
        arr_ptrs = (C.c_void_p * len(ptrs))(*ptrs)
        arr_str = (C.c_uint64 * len(strides))(*strides)
        desc = KernelTaskDesc(arr_args, len(args), len(axis_args) + len(tail), arr_ptrs, arr_str, len(ptrs), 0, 0)
        cycles = self._lib.ptowsp_cuda_run_task(self._h, kernel.encode(), C.byref(desc))
        rc = self._lib.ptowsp_cuda_status(self._h)
        if rc != PTOWSP_OK:
            raise PtoWspCudaError(rc, _last_error())
        return int(cycles)

    def set_stream(self, stream: Any) -> None:
        """Launch on a CUDA stream (torch.cuda.Stream or raw cudaStream_t handle; 0 = default stream)."""
        handle = getattr(stream, "cuda_stream", stream)
        self._lib.ptowsp_cuda_set_stream(self._h, C.c_void_p(int(handle) if handle else None))

    def set_option(self, key: str, value: int) -> None:
        rc = self._lib.ptowsp_cuda_set_option(self._h, key.encode(), int(value))
        if rc != PTOWSP_OK:
            raise PtoWspCudaError(rc, _last_error())

    def timing(self) -> dict:
        t = Timing()
        self._lib.ptowsp_cuda_last_timing(self._h, C.byref(t))
        return {k: getattr(t, k) for k, _ in Timing._fields_}

    def kernel_times(self) -> dict:
        """Per-kernel ``{"launches": n, "ms": t}`` since ``set_option("kernel_events", 1)`` (CUDA events)."""
        return json.loads(self._lib.ptowsp_cuda_kernel_times(self._h).decode())

    def describe(self) -> dict:
        return json.loads(self._lib.ptowsp_cuda_describe(self._h).decode())


def compile_plan(plan: dict, device: int = 0) -> CudaExecutable:
    return CudaExecutable(plan, device)
