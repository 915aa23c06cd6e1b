"""CPU oracle for the PTO-WSP task loop (TEST INFRASTRUCTURE ONLY).

This module restates, in numpy, what the reference CPU-sim artifact does when it
runs a plan (``pto_wsp_b200.plan`` format).  It exists only to check the CUDA
target: the tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import it; the product path never does.

What it restates (reference file:line):

* the generated ``<module>_main`` task loop -- ``emit_workload_cpp_from_ir_ast``
  (``src/python/pto_codegen.cpp:2245-2697``): loop nests over Dense / DenseDyn /
  Ragged axes, Select over CSR, Cond on ScalarExprs, Combine / Sequential,
  slot set / load, per-task ``args`` = axis args + (valid_row, valid_col) per
  tensor param + scalar args (``:2499-2545``), view pointer = base + sum(idx *
  stride) (``:2570-2592``), s3/s4 strides (``:2593-2621``);
* CSP pipelines with CSPT time semantics -- the process threads, channel
  send / recv / close and the max-of-process-clocks result (``:1611-1705``,
  ``:1759-2220``), with the processes interleaved in a fixed order;
* the makespan model ``Scheduler::issue`` (``:1562-1606``) with round-robin /
  key-based worker choice (``:2679-2692``) and the TaskWindow stall;
* the kernel bodies ``emit_kernel_cpp`` (``:470-1241``) as tile-op sequences,
  including which param tiles are pre-loaded (``collect_param_tiles_to_load``
  ``:448-468``), which ops are silently skipped, and the per-op cycle charges of
  ``include/pto/wsp/codegen/abi/ptoisa_bridge.hpp:67-303`` (valid_row*valid_col
  of the destination, M*K*N for TMATMUL, 5*n for TSORT32);
* the built-in custom kernels of this target (paged GQA decode, lightning
  indexer scoring, top-k selection), which the reference expresses only as toy
  examples (``examples/flashinfer_decode/golden.py:7-12``,
  ``examples/deepseek_lightning_indexer/golden.py:6-25``).

Pinned against the reference's own golden values: the example cycle counts
(``examples/*/..._example.py``), the example numpy goldens, and the exact
expectations of ``tests/test_codegen_*.py`` -- see ``tests/test_oracle_pins.py``.
Bit-level TEXP/TRSQRT rounding of the absent pto-isa library is not pinned by
any reference test; numeric checks use the example tolerances.
"""

from __future__ import annotations

import heapq
import math
import struct
from dataclasses import dataclass, field
from typing import Any

import numpy as np

_NP = {"f16": np.float16, "f32": np.float32, "f64": np.float64, "i8": np.int8, "i16": np.int16,
       "i32": np.int32, "i64": np.int64, "u8": np.uint8, "u16": np.uint16, "u32": np.uint32,
       "u64": np.uint64, "bool": np.bool_}

M64 = 0xFFFFFFFFFFFFFFFF


def _u64(v) -> int:
    return int(v, 0) & M64 if isinstance(v, str) else int(v) & M64


def fnv1a_64(s: str) -> int:
    h = 0xCBF29CE484222325
    for b in s.encode("utf-8"):
        h ^= b
        h = (h * 0x100000001B3) & M64
    return h


# ---------------------------------------------------------------------------
# Scheduler (pto_codegen.cpp:1562-1606)
# ---------------------------------------------------------------------------


class Scheduler:
    def __init__(self, num_workers: int, window_tasks: int):
        self.n = num_workers if num_workers else 1
        self.window = window_tasks
        self.issue_time = 0
        self.avail = [0] * self.n
        self.counts = [0] * self.n
        self.in_flight: list[int] = []

    def advance_to(self, t: int) -> None:
        if t > self.issue_time:
            self.issue_time = t
        while self.in_flight and self.in_flight[0] <= self.issue_time:
            heapq.heappop(self.in_flight)

    def issue(self, dur: int, wid: int, ready: int) -> int:
        if wid >= self.n:
            wid = 0
        self.advance_to(ready)
        if self.window > 0:
            while len(self.in_flight) >= self.window:
                self.advance_to(self.in_flight[0])
        start = self.avail[wid] if self.avail[wid] > self.issue_time else self.issue_time
        end = (start + dur) & M64
        self.avail[wid] = end
        self.counts[wid] += 1
        heapq.heappush(self.in_flight, end)
        return end


# ---------------------------------------------------------------------------
# Scalar expressions (include/pto/wsp/ir/scalar_expr.hpp, emitted as C++ by
# emit_scalar_expr_cpp pto_codegen.cpp:207-279): i64/u64/bool with the usual
# C++ arithmetic conversions.
# ---------------------------------------------------------------------------


def _to_i64(v: int) -> int:
    v &= M64
    return v - (1 << 64) if v >> 63 else v


def eval_expr(e: dict, env: "ExprEnv") -> tuple[str, int]:
    op = e["op"]
    if op == "lit":
        return e["type"], (int(e["v"]) & M64 if e["type"] == "u64" else int(e["v"]))
    if op == "axis":
        return "i64", env.axis(_u64(e["id"]))
    if op == "sym":
        return "u64", env.symbol_u64(_u64(e["id"]))
    if op == "tag":
        return "u64", env.symbol_u64(_u64(e["id"]))
    if op == "slot":
        v = env.slot(int(e["i"]))
        if e["type"] == "i64":
            return "i64", _to_i64(v)
        if e["type"] == "bool":
            return "bool", int(v != 0)
        return "u64", v
    if op == "task_param":
        return "u64", env.task_param(int(e["i"]))
    if op == "un":
        t, v = eval_expr(e["a"], env)
        fn = e["fn"]
        if fn == "!":
            return "bool", int(not v)
        if fn == "-":
            return (t, (-v) & M64) if t == "u64" else ("i64", -v)
        return (t, (~v) & M64) if t == "u64" else ("i64", ~v)
    if op == "tern":
        _, c = eval_expr(e["c"], env)
        return eval_expr(e["a"] if c else e["b"], env)
    if op == "cast":
        _, v = eval_expr(e["a"], env)
        ty = e["type"]
        if ty == "bool":
            return "bool", int(v != 0)
        if ty == "u64":
            return "u64", v & M64
        return "i64", _to_i64(v)
    if op == "bin":
        ta, a = eval_expr(e["a"], env)
        tb, b = eval_expr(e["b"], env)
        fn = e["fn"]
        if fn == "&&":
            return "bool", int(bool(a) and bool(b))
        if fn == "||":
            return "bool", int(bool(a) or bool(b))
        unsigned = "u64" in (ta, tb)
        if unsigned:
            a &= M64
            b &= M64
        else:
            a, b = _to_i64(a), _to_i64(b)
        rt = "u64" if unsigned else "i64"
        if fn in ("<", "<=", ">", ">=", "==", "!="):
            r = {"<": a < b, "<=": a <= b, ">": a > b, ">=": a >= b, "==": a == b, "!=": a != b}[fn]
            return "bool", int(r)
        if fn == "+":
            r = a + b
        elif fn == "-":
            r = a - b
        elif fn == "*":
            r = a * b
        elif fn == "/":
            r = int(a / b) if not unsigned else a // b
        elif fn == "%":
            r = a - int(a / b) * b if not unsigned else a % b
        elif fn == "&":
            r = a & b
        elif fn == "|":
            r = a | b
        elif fn == "^":
            r = a ^ b
        elif fn == "<<":
            r = a << (b & 63)
        elif fn == ">>":
            r = (a & M64) >> (b & 63) if unsigned else a >> (b & 63)
        else:
            raise ValueError(f"unknown binary op {fn}")
        return rt, (r & M64) if unsigned else _to_i64(r)
    raise ValueError(f"unknown expr op {op}")


class ExprEnv:
    def __init__(self, rt: "Runtime", axis_env: dict[int, int], task_args: list[int] | None = None):
        self.rt = rt
        self.axis_env = axis_env
        self.task_args = task_args

    def axis(self, aid: int) -> int:
        if aid not in self.axis_env:
            raise ValueError("emit_scalar_expr_cpp: axis_var not in scope")
        return self.axis_env[aid]

    def symbol_u64(self, sid: int) -> int:
        return self.rt.symbols_u64.get(sid, 0)

    def slot(self, i: int) -> int:
        return self.rt.slots[i] if 0 <= i < len(self.rt.slots) else 0

    def task_param(self, i: int) -> int:
        if self.task_args is None:
            raise ValueError("task_param() outside a task")
        return self.task_args[i] if i < len(self.task_args) else 0


# ---------------------------------------------------------------------------
# Tensor views (base + sum(idx*stride), s3/s4)
# ---------------------------------------------------------------------------


def _root(a: np.ndarray) -> np.ndarray:
    r = a
    while isinstance(r.base, np.ndarray):
        r = r.base
    return r


def fma_f32(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """round_f32(a * b + c) with a single rounding (IEEE fusedMultiplyAdd on binary32, round to nearest even).

    The f32 x f32 product is exact in f64; the f64 sum s = RN53(x) of the exact x = a*b + c is turned into
    round-to-odd (truncate toward zero, set the last bit when inexact) from its TwoSum error, and rounding a
    round-to-odd value with at least two extra bits to nearest gives RN24(x) exactly (Boldo & Melquiond,
    "Emulation of FMA and correctly rounded sums: proved algorithms using rounding to odd", IEEE TC 2008).
    """
    a64 = np.asarray(a, dtype=np.float32).astype(np.float64)
    b64 = np.asarray(b, dtype=np.float32).astype(np.float64)
    c64 = np.asarray(c, dtype=np.float32).astype(np.float64)
    p = a64 * b64
    with np.errstate(invalid="ignore", over="ignore"):
        s = p + c64
        bv = s - c64
        err = (c64 - (s - bv)) + (p - bv)  # x - s exactly (TwoSum)
        inexact = np.isfinite(s) & (err != 0)
        t = np.where(inexact & ((err < 0) != (s < 0)), np.nextafter(s, 0.0), s)  # toward zero
        ti = t.view(np.int64)
        t = np.where(inexact, ti | 1, ti).view(np.float64)
        return t.astype(np.float32)


def _elem_strides(a: np.ndarray) -> list[int]:
    return [s // a.itemsize for s in a.strides]


class TensorRef:
    """A tensor argument of the runtime: a numpy array possibly viewing a larger buffer."""

    def __init__(self, arr: np.ndarray):
        self.arr = arr
        root = _root(arr)
        if not root.flags.c_contiguous:
            # a dense buffer in another axis order (e.g. ``transpose(...).astype(...)``, which keeps the permuted
            # layout): address it as the flat run of its memory
            flat = root.ravel(order="K")
            if not np.may_share_memory(flat, root):  # ravel copies when the memory is not one run
                raise ValueError("tensor memory is not one dense buffer")
            root = flat
        self.root = root
        self.itemsize = arr.itemsize
        self.dtype = arr.dtype
        self.base_off = arr.__array_interface__["data"][0] - self.root.__array_interface__["data"][0]
        self.strides = _elem_strides(arr)

    def stride(self, d: int) -> int:
        return self.strides[d] if d < len(self.strides) else 0

    def tile(self, off_elems: int, rows: int, cols: int, s3: int, s4: int) -> np.ndarray:
        # A 2-D strided window at element offset `off_elems` from the tensor base,
        # exactly how GlobalTensor(ptr, Shape(rows, cols), Stride(s3, s4)) reads memory.
        byte_off = self.base_off + off_elems * self.itemsize
        return np.ndarray(shape=(rows, cols), dtype=self.dtype, buffer=self.root, offset=byte_off,
                          strides=(s3 * self.itemsize, s4 * self.itemsize))

    def flat(self, off_elems: int, n: int, stride: int = 1) -> np.ndarray:
        return self.tile(off_elems, 1, n, 0, stride)[0]


@dataclass
class TaskView:
    ref: TensorRef
    off: int  # element offset of the view from the tensor base
    s3: int
    s4: int


def view_of(rt: "Runtime", ta: dict, axis_vals: dict[str, int]) -> TaskView:
    ref = rt.tensors[ta["tensor"]]
    off = 0
    for d, ie in enumerate(ta["index"]):
        v = axis_vals[ie["var"]] if "var" in ie else int(ie["const"])
        off += v * ref.stride(d)
    vr, br = int(ta["view_rank"]), int(ta["base_rank"])
    if vr >= 2:
        s3, s4 = ref.stride(br - vr), ref.stride(br - vr + 1)
    elif vr == 1:
        s3, s4 = 0, ref.stride(br - 1)
    else:
        s3, s4 = 0, 1
    return TaskView(ref, off, s3, s4)


# ---------------------------------------------------------------------------
# Kernel model (emit_kernel_cpp, pto_codegen.cpp:470-1241)
# ---------------------------------------------------------------------------

ROUND_RINT = np.float16  # f32 -> f16 stores use round-to-nearest-even (TCVT CAST_RINT, :959-971)


@dataclass
class KernelModel:
    kd: dict
    values: dict[int, tuple[str, int, int]]
    params: list[dict]
    tensor_params: list[dict]  # in param order, each with value info
    scalar_params: list[dict]
    builtin: str | None
    preload: list[int]
    static_cycles: int | None = None

    @property
    def name(self) -> str:
        return self.kd["name"]


def builtin_name(kd: dict) -> str | None:
    b = kd.get("attrs", {}).get("builtin")
    if b:
        return str(b)
    src = kd.get("attrs", {}).get("cpp_src", "") or ""
    for line in src.splitlines():
        line = line.strip()
        if line.startswith("// ptowsp-builtin:"):
            return line.split(":", 1)[1].strip()
    return None


def build_kernel_model(kd: dict) -> KernelModel:
    values = {int(v[0]): (v[1], int(v[2]), int(v[3])) for v in kd["values"]}
    params, tparams, sparams = [], [], []
    for p in kd["params"]:
        dt, r, c = values[p["id"]]
        info = {"name": p["name"], "id": p["id"], "dtype": dt, "rows": r, "cols": c}
        params.append(info)
        (tparams if r >= 0 else sparams).append(info)
    param_ids = {p["id"] for p in params}
    used: set[int] = set()
    for op in kd["ops"]:
        if op["kind"] in ("Matmul", "Load"):
            continue
        for i, oid in enumerate(op["operands"]):
            if oid not in values or values[oid][1] < 0 or oid not in param_ids:
                continue
            if op["kind"] == "Store" and i == 0:
                continue
            used.add(oid)
    km = KernelModel(kd, values, params, tparams, sparams, builtin_name(kd), sorted(used))
    return km


def _cast_scalar(dtype: str, v: float):
    return _NP[dtype](v)


class _KernelRun:
    """Executes one task of a pto.* kernel and counts CPU-sim cycles."""

    def __init__(self, km: KernelModel, views: list[TaskView], scalars: list[int], execute: bool = True):
        self.km = km
        self.views = {p["id"]: v for p, v in zip(km.tensor_params, views)}
        self.pinfo = {p["id"]: p for p in km.params}
        self.execute = execute
        self.cycles = 0
        self.tiles: dict[int, np.ndarray] = {}
        self.scalar: dict[int, Any] = {}
        for p, raw in zip(km.scalar_params, scalars):
            dt = p["dtype"]
            if dt == "f32":
                self.scalar[p["id"]] = np.float32(struct.unpack("<f", struct.pack("<I", raw & 0xFFFFFFFF))[0])
            elif dt == "i32":
                self.scalar[p["id"]] = np.int32(_to_i64(raw & 0xFFFFFFFF) if raw & 0x80000000 == 0 else (raw & 0xFFFFFFFF) - (1 << 32))
            elif dt == "i64":
                self.scalar[p["id"]] = np.int64(_to_i64(raw))
            elif dt == "bool":
                self.scalar[p["id"]] = raw != 0
        for op in km.kd["ops"]:
            if op["kind"] == "Constant" and op["result"] >= 0:
                dt, r, _ = km.values[op["result"]]
                if r < 0 and "value" in op["attrs"]:
                    self.scalar[op["result"]] = _cast_scalar(dt, float(op["attrs"]["value"]))
        # Store sources take the destination param's valid dims (runtime_dims_by_tile).
        self.store_dims: dict[int, tuple[int, int]] = {}
        for op in km.kd["ops"]:
            if op["kind"] == "Store" and len(op["operands"]) >= 2:
                d = op["operands"][0]
                if d in self.pinfo and self.pinfo[d]["rows"] >= 0:
                    self.store_dims[op["operands"][1]] = (self.pinfo[d]["rows"], self.pinfo[d]["cols"])

    def vdims(self, vid: int) -> tuple[int, int]:
        if vid in self.store_dims:
            return self.store_dims[vid]
        _, r, c = self.km.values[vid]
        return r, c

    def load_param(self, pid: int) -> np.ndarray:
        p = self.pinfo[pid]
        v = self.views[pid]
        t = v.ref.tile(v.off, p["rows"], p["cols"], v.s3, v.s4) if self.execute else None
        return np.array(t, dtype=_NP[p["dtype"]]) if self.execute else None

    def run(self) -> int:
        km = self.km
        for pid in km.preload:
            self.tiles[pid] = self.load_param(pid)
            self.cycles += self.pinfo[pid]["rows"] * self.pinfo[pid]["cols"]
        local = set()
        for op in km.kd["ops"]:
            rid = op["result"]
            if rid >= 0 and rid not in self.pinfo and km.values.get(rid, ("", -1, -1))[1] >= 0:
                local.add(rid)
        for op in km.kd["ops"]:
            self._op(op, local)
        return self.cycles

    def _is_tile(self, vid: int) -> bool:
        return vid in self.tiles

    def _op(self, op: dict, local: set[int]) -> None:
        k = op["kind"]
        rid = op["result"]
        ops = op["operands"]
        km = self.km
        ex = self.execute
        if k == "Load":
            if rid < 0 or not ops or ops[0] not in self.pinfo or rid not in local:
                return
            self.tiles[rid] = self.load_param(ops[0])
            r, c = self.vdims(rid)
            self.cycles += r * c
            return
        if k == "Matmul":
            if rid < 0 or len(ops) < 2 or rid not in local:
                return
            a_id, b_id = ops[0], ops[1]

            def shape_dtype(oid):
                if oid in self.pinfo:
                    p = self.pinfo[oid]
                    return (p["rows"], p["cols"]), p["dtype"], True
                if oid in local:
                    dt, r, c = km.values[oid]
                    return (r, c), dt, False
                return None, None, False

            (ash, adt, ap), (bsh, bdt, bp) = shape_dtype(a_id), shape_dtype(b_id)
            if ash is None or bsh is None or ash[1] != bsh[0]:
                return
            rdt = km.values[rid][0]
            if not ((adt == bdt == "f32" and rdt == "f32") or (adt == bdt == "f16" and rdt == "f32")):
                return
            m, kk = ash
            n = bsh[1]
            self.cycles += m * kk  # TLOAD / TMOV into TileLeft
            self.cycles += kk * n  # TLOAD / TMOV into TileRight
            self.cycles += m * kk * n  # TMATMUL
            if ex:
                a = self.load_param(a_id) if ap else self.tiles[a_id]
                b = self.load_param(b_id) if bp else self.tiles[b_id]
                # sequential-k f32 accumulation, one fused multiply-add per step (separately rounded products
                # would fail the reference's llama example check on one element where res1 + mlp cancels:
                # error 1.3e-6 against its 1.04e-6 bound; f16 inputs give exact products either way)
                acc = np.zeros((m, n), dtype=np.float32)
                a32 = np.asarray(a, dtype=np.float32)
                b32 = np.asarray(b, dtype=np.float32)
                for kk_i in range(kk):
                    acc = fma_f32(a32[:, kk_i, None], b32[None, kk_i, :], acc)
                self.tiles[rid] = acc
            else:
                self.tiles[rid] = None
            # acc -> vec TMOV when a non-matmul, non-store op consumes it
            for o2 in km.kd["ops"]:
                if o2["kind"] in ("Matmul", "Store"):
                    continue
                if rid in o2["operands"]:
                    r, c = self.vdims(rid)
                    self.cycles += r * c
                    break
            return
        if k == "Store":
            if len(ops) < 2 or ops[0] not in self.pinfo or self.pinfo[ops[0]]["rows"] < 0:
                return
            dst, src = ops[0], ops[1]
            # local tiles = op results plus pre-loaded param tiles
            if (src not in local and src not in km.preload) or src not in self.tiles:
                return
            p = self.pinfo[dst]
            sdt = km.values[src][0]
            if p["dtype"] != sdt and not (p["dtype"] == "f16" and sdt == "f32"):
                return
            sr, sc = p["rows"], p["cols"]
            if p["dtype"] != sdt:
                self.cycles += sr * sc  # TCVT
            self.cycles += sr * sc  # TSTORE (src tile valid dims = dst param dims)
            if ex:
                v = self.views[dst]
                t = v.ref.tile(v.off, sr, sc, v.s3, v.s4)
                t[...] = np.asarray(self.tiles[src])[:sr, :sc].astype(_NP[p["dtype"]])
            return
        if k in ("Add", "Sub", "Mul", "Div", "Max", "Min"):
            if rid < 0 or len(ops) != 2 or rid not in local:
                return
            a_id, b_id = ops
            a_s, b_s = a_id in self.scalar, b_id in self.scalar
            dt = km.values[rid][0]
            r, c = self.vdims(rid)
            if a_s ^ b_s:
                tid = b_id if a_s else a_id
                sid = a_id if a_s else b_id
                if tid not in self.tiles:
                    return
                s = self.scalar[sid]
                t = self.tiles[tid]
                if k == "Sub" and a_s:
                    return  # "scalar - tile not supported" (pto_codegen.cpp:1040-1041)
                self.cycles += r * c
                if ex:
                    t = np.asarray(t, dtype=_NP[dt])
                    s = _NP[dt](s)
                    if k == "Add":
                        out = t + s
                    elif k == "Mul":
                        out = t * s
                    elif k == "Div":
                        out = t / s if b_s else s / t
                    elif k == "Sub":
                        out = t - s
                    elif k == "Max":
                        out = np.maximum(t, s)
                    else:
                        out = np.minimum(t, s)
                    self.tiles[rid] = out.astype(_NP[dt])
                else:
                    self.tiles[rid] = None
                return
            if a_id not in self.tiles or b_id not in self.tiles:
                return
            ash = km.values[a_id][1:] if a_id in km.values else None
            bsh = km.values[b_id][1:] if b_id in km.values else None
            sr, sc = km.values[rid][1:]
            mode = None
            if ash == (sr, sc) and bsh == (sr, sc):
                mode = "full"
            elif ash == (sr, sc) and (bsh == (sr, 1) or bsh == (1, sr)):
                mode = "row"
            elif k in ("Sub", "Mul", "Div") and ash == (sr, sc) and (bsh == (1, sc) or bsh == (sc, 1)):
                mode = "col"
            if mode is None:
                return  # "broadcast pattern unsupported" -- no code, no cycles
            self.cycles += r * c
            if ex:
                a = np.asarray(self.tiles[a_id], dtype=_NP[dt])
                b = np.asarray(self.tiles[b_id], dtype=_NP[dt])
                if mode == "row":
                    b = b.reshape(-1)[:sr].reshape(sr, 1)
                elif mode == "col":
                    b = b.reshape(-1)[:sc].reshape(1, sc)
                fn = {"Add": np.add, "Sub": np.subtract, "Mul": np.multiply, "Div": np.divide,
                      "Max": np.maximum, "Min": np.minimum}[k]
                self.tiles[rid] = fn(a, b).astype(_NP[dt])
            else:
                self.tiles[rid] = None
            return
        if k in ("Exp", "Rsqrt"):
            if rid < 0 or len(ops) != 1 or rid not in local or ops[0] not in self.tiles:
                return
            r, c = self.vdims(rid)
            self.cycles += r * c
            if ex:
                x = np.asarray(self.tiles[ops[0]], dtype=np.float32)
                with np.errstate(divide="ignore", over="ignore", invalid="ignore"):
                    y = np.exp(x) if k == "Exp" else (np.float32(1.0) / np.sqrt(x))
                self.tiles[rid] = y.astype(_NP[km.values[rid][0]])
            else:
                self.tiles[rid] = None
            return
        if k == "IotaU32":
            if rid < 0 or rid not in local:
                return
            r, c = km.values[rid][1:]
            if r != 1:
                return
            self.tiles[rid] = np.arange(c, dtype=np.uint32).reshape(1, c) if ex else None
            return
        if k == "TSort32":
            if rid < 0 or len(ops) != 2 or rid not in local or ops[0] not in self.tiles or ops[1] not in self.tiles:
                return
            sr, sc = self.vdims(ops[0]) if ops[0] in self.store_dims else km.values[ops[0]][1:]
            if ops[0] in self.pinfo:
                sr, sc = self.pinfo[ops[0]]["rows"], self.pinfo[ops[0]]["cols"]
            self.cycles += 5 * sr * sc
            if ex:
                s = np.asarray(self.tiles[ops[0]], dtype=np.float32).reshape(-1)
                idx = np.asarray(self.tiles[ops[1]]).reshape(-1)
                order = np.lexsort((np.arange(s.size), -s.astype(np.float64)))
                out = np.zeros(2 * s.size, dtype=np.float32)
                out[0::2] = s[order]
                out[1::2] = idx[order].astype(np.float32)
                r2, c2 = km.values[rid][1:]
                full = np.zeros(r2 * c2, dtype=np.float32)
                full[: min(out.size, full.size)] = out[: full.size]
                self.tiles[rid] = full.reshape(r2, c2)
            else:
                self.tiles[rid] = None
            return
        if k == "ExtractTopkIndices":
            if rid < 0 or len(ops) != 1 or rid not in local or ops[0] not in self.tiles:
                return
            kk = int(op["attrs"].get("k", 0)) or km.values[rid][2]
            if ex:
                pairs = np.asarray(self.tiles[ops[0]], dtype=np.float32).reshape(-1)
                r2, c2 = km.values[rid][1:]
                out = np.zeros(r2 * c2, dtype=_NP[km.values[rid][0]])
                out[:kk] = pairs[1: 2 * kk: 2].astype(np.int32)
                self.tiles[rid] = out.reshape(r2, c2)
            else:
                self.tiles[rid] = None
            return
        if k in ("RowSum", "RowMax", "RowMean"):
            if rid < 0 or len(ops) != 1 or rid not in local or ops[0] not in self.tiles:
                return
            r, c = self.vdims(rid)
            self.cycles += r * c * (2 if k == "RowMean" else 1)
            if ex:
                x = np.asarray(self.tiles[ops[0]], dtype=np.float32)
                if k == "RowMax":
                    y = x.max(axis=1, keepdims=True)
                else:
                    y = np.zeros((x.shape[0], 1), dtype=np.float32)
                    for j in range(x.shape[1]):  # sequential column accumulation
                        y[:, 0] += x[:, j]
                    if k == "RowMean":
                        y = y / np.float32(km.values[ops[0]][2])
                self.tiles[rid] = y.astype(_NP[km.values[rid][0]])
            else:
                self.tiles[rid] = None
            return
        # Unhandled op kind: cycles += static r*c of the result (pto_codegen.cpp:1223-1231)
        if rid >= 0 and rid in km.values and km.values[rid][1] >= 0:
            self.cycles += km.values[rid][1] * km.values[rid][2]


# ---------------------------------------------------------------------------
# Built-in custom kernels of the cuda_sm100a target
# ---------------------------------------------------------------------------


def builtin_run(name: str, km: KernelModel, views: list[TaskView], axis_args: list[int], scalars: list[int],
                execute: bool) -> int:
    """Numpy restatement of the target's built-in custom kernels; returns modeled cycles."""
    byid = {p["id"]: (p, v) for p, v in zip(km.tensor_params, views)}
    tp = km.tensor_params
    if name == "paged_decode_gqa":
        # params: q[G,D] f16, k_cache, v_cache (pages x page_size x KVH x D, f16),
        #         page_table[1,maxp] i32, kv_len[1,1] i32, out[G,D] f16.
        # axis args: (request, kv_head).  scalars: page_size, num_kv_heads.
        q_p, k_p, v_p, pt_p, len_p, o_p = [byid[p["id"]] for p in tp]
        G, D = q_p[0]["rows"], q_p[0]["cols"]
        page_size, kvh = int(scalars[0]), int(scalars[1])
        h = int(axis_args[1])
        L = int(len_p[1].ref.flat(len_p[1].off, 1)[0])
        L = min(L, pt_p[0]["cols"] * page_size)
        # model charge: shape-static, with the page-table capacity as the length
        Ls = pt_p[0]["cols"] * page_size
        cycles = G * D + 2 * Ls * D + G * D * Ls + 5 * G * Ls + 2 * G + G * Ls * D + G * D
        if not execute or L <= 0:
            if execute and L <= 0:
                o_p[1].ref.tile(o_p[1].off, G, D, o_p[1].s3, o_p[1].s4)[...] = 0
            return cycles
        npages = (L + page_size - 1) // page_size
        pages = pt_p[1].ref.flat(pt_p[1].off, npages, max(pt_p[1].s4, 1)).astype(np.int64)
        q = q_p[1].ref.tile(q_p[1].off, G, D, q_p[1].s3, q_p[1].s4).astype(np.float64)
        kc, vc = k_p[1], v_p[1]
        # cache layout [pages, page_size, KVH, D]: s3 = page stride, s4 = token stride
        tok = np.arange(L)
        rows_off = pages[tok // page_size] * kc.s3 + (tok % page_size) * kc.s4 + h * D
        K = np.stack([kc.ref.flat(kc.off + int(o), D) for o in rows_off]).astype(np.float64)
        rows_off_v = pages[tok // page_size] * vc.s3 + (tok % page_size) * vc.s4 + h * D
        V = np.stack([vc.ref.flat(vc.off + int(o), D) for o in rows_off_v]).astype(np.float64)
        s = (q @ K.T) * (1.0 / math.sqrt(D))
        s = s - s.max(axis=1, keepdims=True)
        w = np.exp(s)
        w = w / w.sum(axis=1, keepdims=True)
        out = w @ V
        o_p[1].ref.tile(o_p[1].off, G, D, o_p[1].s3, o_p[1].s4)[...] = out.astype(np.float16)
        return cycles
    if name == "lightning_indexer_score":
        # params: q[Q*H, D] f16, k[T, D] f16, w[Q, H] f32, scores[Q, T] f32
        q_p, k_p, w_p, s_p = [byid[p["id"]] for p in tp]
        QH, D = q_p[0]["rows"], q_p[0]["cols"]
        T = k_p[0]["rows"]
        Q, H = w_p[0]["rows"], w_p[0]["cols"]
        cycles = QH * D + T * D + QH * D * T + 2 * QH * T + Q * T
        if not execute:
            return cycles
        q = q_p[1].ref.tile(q_p[1].off, QH, D, q_p[1].s3, q_p[1].s4).astype(np.float32)
        k = k_p[1].ref.tile(k_p[1].off, T, D, k_p[1].s3, k_p[1].s4).astype(np.float32)
        w = w_p[1].ref.tile(w_p[1].off, Q, H, w_p[1].s3, w_p[1].s4).astype(np.float64)
        dots = (q.astype(np.float64) @ k.astype(np.float64).T).reshape(Q, H, T)
        sc = np.einsum("qh,qht->qt", w, np.maximum(dots, 0.0))
        s_p[1].ref.tile(s_p[1].off, Q, T, s_p[1].s3, s_p[1].s4)[...] = sc.astype(np.float32)
        return cycles
    if name == "topk_select":
        # params: scores[1, N] f32, out[1, K] i32.  Stable: score desc, ties -> lower index.
        s_p, o_p = [byid[p["id"]] for p in tp]
        N, K = s_p[0]["cols"], o_p[0]["cols"]
        cycles = N + 5 * N + K
        if not execute:
            return cycles
        s = s_p[1].ref.flat(s_p[1].off, N, max(s_p[1].s4, 1)).astype(np.float32)
        order = stable_topk(s, K)
        o_p[1].ref.flat(o_p[1].off, K, max(o_p[1].s4, 1))[...] = order.astype(np.int32)
        return cycles
    raise ValueError(f"unknown built-in kernel {name!r}")


def stable_topk(scores: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest scores, ties -> lower index (golden.py:7-24 rule)."""
    s = np.asarray(scores, dtype=np.float32)
    # order-preserving key: larger float -> larger key; -0.0 and +0.0 compare equal
    bits = s.view(np.uint32).astype(np.uint64)
    neg = (bits >> 31) == 1
    key = np.where(neg, (~bits) & 0xFFFFFFFF, bits | 0x80000000)
    key = np.where(s == 0, np.uint64(0x80000000), key)
    order = np.lexsort((np.arange(s.size), -key.astype(np.int64)))
    return order[:k]


# ---------------------------------------------------------------------------
# Runtime (the <module>_main walk)
# ---------------------------------------------------------------------------


@dataclass
class Runtime:
    tensors: list[TensorRef]
    axis_sizes: dict[str, int]
    symbols_u64: dict[int, int]
    symbols_ptr: dict[int, np.ndarray]
    slots: list[int] = field(default_factory=lambda: [0] * 256)


class CpuSim:
    """Runs a plan the way the reference CPU-sim artifact would."""

    def __init__(self, plan: dict):
        self.plan = plan
        self.models = {k["name"]: build_kernel_model(k) for k in plan["kernels"]}
        sch = plan.get("schedule") or {}
        disp = sch.get("dispatch")
        tw = sch.get("task_window")
        self.num_workers = 1
        if disp and disp.get("num_targets", 0) > 0:
            self.num_workers = int(disp["num_targets"])
        elif sch.get("streams", 0) > 0:
            self.num_workers = int(sch["streams"])
        self.window = 0
        if tw and tw.get("unit") == "tasks" and tw.get("overflow", "stall") == "stall":
            self.window = max(int(tw["size"]), 0)
        self.dispatch = disp
        self.task_log: list[tuple[str, dict[str, int], int]] = []

    def run(self, arrays: list[np.ndarray], axis_sizes: dict[str, int] | None = None,
            symbols_u64: dict[int, int] | None = None, symbols_ptr: dict[int, np.ndarray] | None = None,
            execute: bool = True, log_tasks: bool = False) -> int:
        rt = Runtime([TensorRef(a) for a in arrays], dict(axis_sizes or {}), dict(symbols_u64 or {}),
                     dict(symbols_ptr or {}))
        self.rt = rt
        self.execute = execute
        self.log_tasks = log_tasks
        self.task_log = []
        self.sched = Scheduler(self.num_workers, self.window)
        self.rr = 0
        return self._node(self.plan["body"], 0, {}, {})

    # axis_env: var-id -> value (for scalar exprs); vals: var name -> value (for views)
    def _bounds(self, axis: dict, var: str) -> int:
        k = axis["kind"]
        if k == "dense":
            return int(axis["size"])
        if k == "dense_dyn":
            return int(self.rt.axis_sizes.get(var, 0))
        if k == "ragged":
            outer = self.rt.symbols_u64.get(_u64(axis["outer_sym"]), 0)
            lens = self.rt.symbols_ptr.get(_u64(axis["lengths_sym"]))
            if lens is None:
                return 0
            return int(np.asarray(lens, dtype=np.int64).reshape(-1)[: int(outer)].sum())
        raise ValueError(f"Unsupported axis kind {k}")

    def _node(self, n: dict, ready: int, axis_env: dict[int, int], vals: dict[str, int]) -> int:
        k = n["kind"]
        if k == "slot_set":
            self.rt.slots[int(n["slot"])] = _u64(n["value"])
            return ready
        if k == "slot_load":
            v = view_of(self.rt, n["tensor_arg"], vals)
            x = v.ref.tile(v.off, 1, 1, 0, 1)  # base pointer of the view
            e = v.ref.flat(v.off + int(n["row"]) * v.s3 + int(n["col"]) * v.s4, 1)[0]
            del x
            self.rt.slots[int(n["slot"])] = int(e) & M64
            return ready
        if k in ("parallel_for", "for_each"):
            var = n["var"]
            vid = fnv1a_64(var)
            ub = self._bounds(n["axis"], var)
            done = ready
            cur = ready
            for i in range(ub):
                env2 = dict(axis_env)
                env2[vid] = i
                vals2 = dict(vals)
                vals2[var] = i
                if k == "parallel_for":
                    done = max(done, self._node(n["body"], ready, env2, vals2))
                else:
                    cur = self._node(n["body"], cur, env2, vals2)
            return done if k == "parallel_for" else cur
        if k == "select":
            outer = self.rt.symbols_u64.get(_u64(n["outer_sym"]), 0)
            indptr = self.rt.symbols_ptr.get(_u64(n["indptr_sym"]))
            indices = self.rt.symbols_ptr.get(_u64(n["indices_sym"]))
            nnz = int(np.asarray(indptr).reshape(-1)[int(outer)]) if indptr is not None else 0
            done = ready
            var = n["var"]
            for p in range(nnz):
                idx = int(np.asarray(indices).reshape(-1)[p]) if indices is not None else 0
                env2 = dict(axis_env)
                env2[fnv1a_64(var)] = idx
                vals2 = dict(vals)
                vals2[var] = idx
                done = max(done, self._node(n["body"], ready, env2, vals2))
            return done
        if k == "cond":
            _, c = eval_expr(n["pred"], ExprEnv(self.rt, axis_env))
            return self._node(n["then"] if c else n["else"], ready, axis_env, vals)
        if k == "combine":
            done = ready
            for ch in n["children"]:
                done = max(done, self._node(ch, ready, axis_env, vals))
            return done
        if k == "sequential":
            cur = ready
            for ch in n["children"]:
                cur = self._node(ch, cur, axis_env, vals)
            return cur
        if k == "task":
            return self._task(n, ready, axis_env, vals)
        if k == "pipeline":
            return max(ready, self._pipeline(n))
        raise ValueError(f"Unhandled workload node kind {k}")

    # ---- CSP pipelines: CSPT time semantics (pto_codegen.cpp:1611-1705 channel, :1759-2220 processes) ----
    # Each process has its own clock; a task adds its cycle charge to it; a channel carries (token, send time);
    # a receive raises the receiver's clock to send time + latency and records it as the channel's last pop
    # time; a sender that waited for room (or a rendezvous) raises its clock to the last pop time.  The
    # pipeline's result is the largest clock.  The reference runs the processes as threads; this restatement
    # interleaves them deterministically: the first runnable process in declaration order runs until its next
    # channel operation completes (then the choice is made again) or blocks.

    def _pipeline(self, n: dict) -> int:
        lat = self.rt.symbols_u64.get(fnv1a_64("__pto_wsp_channel_latency_cycles"), 0)
        names = {c["name"]: i for i, c in enumerate(n["channels"])}
        chans = [{"cap": max(0, int(c["capacity"])), "buf": [], "closed": False, "rw": False, "has": False,
                  "rdv": (0, 0), "last_pop": 0} for c in n["channels"]]
        procs = []
        for p in n["processes"]:
            st = {"t": 0, "blocked": None, "done": False}
            procs.append((p, st, self._cspt(p["body"], st, chans, names, lat, {}, {})))

        def wake(kind: str, ci: int) -> None:
            for _, q, _ in procs:
                if q["blocked"] == (kind, ci):
                    q["blocked"] = None

        self._cspt_wake = wake
        while True:
            pick = next((i for i, (_, st, _) in enumerate(procs) if not st["done"] and st["blocked"] is None), None)
            if pick is None:
                if all(st["done"] for _, st, _ in procs):
                    break
                raise RuntimeError("CSP pipeline deadlock: every unfinished process waits on a channel")
            p, st, gen = procs[pick]
            try:
                next(gen)
            except StopIteration:
                st["done"] = True
                for name in p["produces"]:
                    ci = names[name]
                    chans[ci]["closed"] = True
                    wake("send", ci)
                    wake("recv", ci)
        return max((st["t"] for _, st, _ in procs), default=0)

    def _cspt(self, n: dict, st: dict, chans: list, names: dict, lat: int, axis_env: dict, vals: dict):
        k = n["kind"]
        if k in ("slot_set", "slot_load"):
            self._node(n, 0, axis_env, vals)
        elif k == "task":
            st["t"] += self._task_run(n, axis_env, vals)[0]
        elif k in ("parallel_for", "for_each"):
            if n["axis"]["kind"] not in ("dense", "dense_dyn"):
                raise ValueError("CSPT codegen: unsupported axis kind in loop")
            var = n["var"]
            for i in range(self._bounds(n["axis"], var)):
                yield from self._cspt(n["body"], st, chans, names, lat, {**axis_env, fnv1a_64(var): i},
                                      {**vals, var: i})
        elif k == "cond":
            _, c = eval_expr(n["pred"], ExprEnv(self.rt, axis_env))
            yield from self._cspt(n["then"] if c else n["else"], st, chans, names, lat, axis_env, vals)
        elif k in ("combine", "sequential"):
            for ch in n["children"]:
                yield from self._cspt(ch, st, chans, names, lat, axis_env, vals)
        elif k == "send":
            task = n["value"]
            dur, args = self._task_run(task, axis_env, vals)
            st["t"] += dur
            token = args[0] if task["axis_args"] else 0
            yield from self._send(chans, names[n["channel"]], token, st)
        elif k == "consume":
            ci = names[n["channel"]]
            var = n["var"]
            while True:
                got, tok = yield from self._recv(chans, ci, lat, st)
                if not got:
                    break
                yield from self._cspt(n["body"], st, chans, names, lat, {**axis_env, fnv1a_64(var): tok},
                                      {**vals, var: tok})
        else:
            raise ValueError("CSPT codegen: unsupported node kind in process body")

    def _send(self, chans: list, ci: int, token: int, st: dict):
        c = chans[ci]
        if c["cap"] > 0:
            while not c["closed"] and len(c["buf"]) >= c["cap"]:
                st["blocked"] = ("send", ci)
                yield
                st["t"] = max(st["t"], c["last_pop"])
            if not c["closed"]:
                c["buf"].append((token, st["t"]))
                self._cspt_wake("recv", ci)
            yield
            return
        while not c["closed"] and not c["rw"]:  # rendezvous: a receiver must be waiting
            st["blocked"] = ("send", ci)
            yield
        if c["closed"]:
            yield
            return
        c["rdv"] = (token, st["t"])
        c["has"] = True
        self._cspt_wake("recv", ci)
        while not c["closed"] and c["has"]:
            st["blocked"] = ("send", ci)
            yield
        st["t"] = max(st["t"], c["last_pop"])
        yield

    def _recv(self, chans: list, ci: int, lat: int, st: dict):
        c = chans[ci]
        if c["cap"] > 0:
            while not c["buf"] and not c["closed"]:
                st["blocked"] = ("recv", ci)
                yield
            if not c["buf"]:
                return False, 0
            tok, ts = c["buf"].pop(0)
        else:
            c["rw"] = True
            self._cspt_wake("send", ci)
            while not c["closed"] and not c["has"]:
                st["blocked"] = ("recv", ci)
                yield
            c["rw"] = False
            if not c["has"]:
                return False, 0
            (tok, ts), c["has"] = c["rdv"], False
        st["t"] = max(st["t"], ts + lat)
        c["last_pop"] = st["t"]
        self._cspt_wake("send", ci)
        yield
        return True, tok

    def _arg(self, a: dict, vals: dict[str, int]) -> int:
        if "var" in a:
            return int(vals[a["var"]]) & M64
        if "sym" in a:
            return self.rt.symbols_u64.get(_u64(a["sym"]), 0)
        return _u64(a["u64"])

    def _task(self, n: dict, ready: int, axis_env: dict[int, int], vals: dict[str, int]) -> int:
        dur, args = self._task_run(n, axis_env, vals)
        disp = self.dispatch
        if not disp:
            wid = 0
        elif disp["policy"] in ("round_robin", "work_steal"):
            wid = self.rr % self.sched.n
            self.rr += 1
        else:
            if disp.get("key") is None:
                raise ValueError("dispatch policy requires ScalarExpr key")
            _, key = eval_expr(disp["key"], ExprEnv(self.rt, axis_env, args))
            wid = (key & M64) % self.sched.n
        return self.sched.issue(dur, int(wid), ready)

    def _task_run(self, n: dict, axis_env: dict[int, int], vals: dict[str, int]) -> tuple[int, list[int]]:
        """Run one task on the arrays; (its cycle charge, its u64 args)."""
        km = self.models.get(n["kernel"])
        if km is None:
            raise ValueError(f"Missing kernel def for task: {n['kernel']}")
        user_axis = [self._arg(a, vals) for a in n["axis_args"]]
        tail = []
        for p in km.tensor_params:
            tail += [p["rows"], p["cols"]]
        scal = [self._arg(a, vals) for a in n["scalar_args"]]
        args = user_axis + tail + scal
        by_param = {ta["param"]: ta for ta in n["tensor_args"]}
        views = []
        for p in km.tensor_params:
            if p["name"] not in by_param:
                raise ValueError(f"Missing tensor arg for param: {p['name']}")
            views.append(view_of(self.rt, by_param[p["name"]], vals))
        if km.builtin:
            dur = builtin_run(km.builtin, km, views, user_axis, scal, self.execute)
        else:
            if not self.execute and km.static_cycles is not None:
                dur = km.static_cycles
            else:
                dur = _KernelRun(km, views, scal, self.execute).run()
                if not self.execute:
                    km.static_cycles = dur
        if self.log_tasks:
            self.task_log.append((n["kernel"], dict(vals), dur))
        return dur, args


def run_plan(plan: dict, arrays: list[np.ndarray], **kw) -> int:
    return CpuSim(plan).run(arrays, **kw)


def kernel_cycles(plan: dict, kernel: str) -> int:
    """Per-task cycle charge of a pto.* kernel (shape-static)."""
    km = build_kernel_model(next(k for k in plan["kernels"] if k["name"] == kernel))
    views = [None] * len(km.tensor_params)
    return _KernelRun(km, views, [0] * len(km.scalar_params), execute=False).run()


class OracleExecutable:
    """``CodegenExecutable``-shaped wrapper (run_with_symbols) around :class:`CpuSim`."""

    so_path = "<oracle>"

    def __init__(self, plan: dict):
        self.plan = plan
        self.entrypoint = f"{plan.get('name', 'main')}_main"
        self.sim = CpuSim(plan)

    def run_with_symbols(self, arrays, axis_sizes, symbols_u64, symbols_ptr) -> int:
        return self.sim.run(list(arrays), axis_sizes, symbols_u64, symbols_ptr)

    def run(self, arrays, axis_sizes) -> int:
        return self.run_with_symbols(arrays, axis_sizes, {}, {})
