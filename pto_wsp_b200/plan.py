"""Portable workload plans: the reference's codegen ``ir::Module`` as plain JSON.

The reference lowers a ``@workload`` into a C++ ``ir::Module`` with codegen
attachments (``python/pto_wsp/ir_bridge.py:112-139``) and hands it to
``compile_codegen`` (``src/python/pto_codegen.cpp:3352-3434``).  The CUDA target
does not emit C++ per module; instead the module is serialised into a *plan*
(JSON, format ``ptowsp-plan/1``) that the C-ABI runtime (``ptowsp_cuda_compile``)
parses, lowers into launch groups and executes.  A plan carries exactly what the
reference emitter reads from the module:

* ``tensors``   -- ``CodegenTensorInfo`` (dtype, shape) per tensor id
  (``include/pto/wsp/ir/codegen.hpp:42-45``);
* ``kernels``   -- ``CodegenKernelDef`` (params, values, ops, attrs)
  (``include/pto/wsp/ir/codegen.hpp:51-77``);
* ``body``      -- the workload tree: ParallelFor / ForEach over Dense, DenseDyn
  and Ragged axes, Select, Cond, Combine, Sequential, Task, slot set/load
  (walked by ``emit_workload_cpp_from_ir_ast``, ``src/python/pto_codegen.cpp:2245-2697``);
* ``schedule``  -- dispatch policy + task window
  (``src/python/pto_codegen.cpp:1500-1560``).

``module_to_plan`` reads a live pybind ``ir::Module`` (needs the reference's
``pto_ir_cpp``); everything else here is plain Python so plans can be stored as
fixtures and replayed on a machine without the reference installed.
"""

from __future__ import annotations

import json
import re
from typing import Any

PLAN_FORMAT = "ptowsp-plan/1"

_DTYPE_NAMES = {
    "F16": "f16", "BF16": "bf16", "F32": "f32", "F64": "f64", "I8": "i8", "I16": "i16",
    "I32": "i32", "I64": "i64", "U8": "u8", "U16": "u16", "U32": "u32", "U64": "u64",
    "Bool": "bool", "BOOL": "bool",
}

DTYPE_BYTES = {"f16": 2, "bf16": 2, "f32": 4, "f64": 8, "i8": 1, "i16": 2, "i32": 4, "i64": 8,
               "u8": 1, "u16": 2, "u32": 4, "u64": 8, "bool": 1}


def fnv1a_64(s: str) -> int:
    """Stable symbol / axis id (``program.py:358``, ``pto_codegen.cpp:118-125``)."""
    h = 0xCBF29CE484222325
    for b in s.encode("utf-8"):
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def _dtype(dt: Any) -> str:
    name = getattr(dt, "name", None) or str(dt).split(".")[-1]
    if name in _DTYPE_NAMES:
        return _DTYPE_NAMES[name]
    low = str(name).lower()
    if low in DTYPE_BYTES:
        return low
    raise ValueError(f"unsupported dtype in plan: {dt!r}")


def _hex(v: int) -> str:
    return "0x%x" % (int(v) & 0xFFFFFFFFFFFFFFFF)


# ---------------------------------------------------------------------------
# Scalar expressions
# ---------------------------------------------------------------------------
#
# The pybind layer exposes ScalarExpr nodes only through ``print()`` (C++ form,
# ``include/pto/wsp/ir/scalar_expr.hpp:85-260``) and dispatch keys only through
# their Python debug string (``python/pto_wsp/scalar_expr.py:80-101``).  Both
# grammars are fully parenthesised, so one small recursive-descent parser reads
# either into the plan's expression dicts.

_TOKEN = re.compile(
    r"\s*(?:(0x[0-9a-fA-F]+u?)|(\d+u?)|(\|\||&&|<<|>>|<=|>=|==|!=|[-+*/%&|^<>!~?:()\[\],.])|([A-Za-z_][A-Za-z_0-9]*))"
)

_BIN_PREC = [
    ["||"], ["&&"], ["|"], ["^"], ["&"], ["==", "!="], ["<", "<=", ">", ">="], ["<<", ">>"], ["+", "-"],
    ["*", "/", "%"],
]


def _tokenize(text: str) -> list[str]:
    out = []
    pos = 0
    text = text.strip()
    while pos < len(text):
        m = _TOKEN.match(text, pos)
        if not m or m.end() == pos:
            raise ValueError(f"cannot tokenize scalar expr {text!r} at {pos}")
        tok = next(g for g in m.groups() if g is not None)
        out.append(tok)
        pos = m.end()
    return out


class _ExprParser:
    def __init__(self, text: str):
        self.toks = _tokenize(text)
        self.i = 0
        self.text = text

    def peek(self) -> str | None:
        return self.toks[self.i] if self.i < len(self.toks) else None

    def take(self, expect: str | None = None) -> str:
        tok = self.peek()
        if tok is None or (expect is not None and tok != expect):
            raise ValueError(f"bad scalar expr {self.text!r}: expected {expect!r}, got {tok!r}")
        self.i += 1
        return tok

    def parse(self) -> dict:
        e = self.expr()
        if self.peek() is not None:
            raise ValueError(f"trailing tokens in scalar expr {self.text!r}")
        return e

    def expr(self) -> dict:
        c = self.binary(0)
        if self.peek() == "?":
            self.take("?")
            a = self.expr()
            self.take(":")
            b = self.expr()
            return {"op": "tern", "c": c, "a": a, "b": b}
        return c

    def binary(self, level: int) -> dict:
        if level >= len(_BIN_PREC):
            return self.unary()
        lhs = self.binary(level + 1)
        while self.peek() in _BIN_PREC[level]:
            fn = self.take()
            rhs = self.binary(level + 1)
            lhs = {"op": "bin", "fn": fn, "a": lhs, "b": rhs}
        return lhs

    def unary(self) -> dict:
        tok = self.peek()
        if tok in ("!", "-", "~"):
            self.take()
            return {"op": "un", "fn": tok, "a": self.unary()}
        return self.atom()

    def _int_arg(self) -> int:
        self.take("(")
        tok = self.take()
        self.take(")")
        return int(tok.rstrip("u"), 0)

    def atom(self) -> dict:
        tok = self.take()
        if tok == "(":
            # cast "(type)(expr)" or parenthesised expr
            if self.peek() in ("bool", "i64", "u64") and self.i + 1 < len(self.toks) and self.toks[self.i + 1] == ")":
                ty = self.take()
                self.take(")")
                self.take("(")
                inner = self.expr()
                self.take(")")
                return {"op": "cast", "type": ty, "a": inner}
            if self.peek() in ("!", "-", "~") and self.i + 1 < len(self.toks) and self.toks[self.i + 1] not in (")",):
                # python debug unary form "(op expr)" or C++ "(!expr)"
                fn = self.take()
                inner = self.expr()
                self.take(")")
                return {"op": "un", "fn": fn, "a": inner}
            e = self.expr()
            self.take(")")
            return e
        if tok in ("true", "True"):
            return {"op": "lit", "type": "bool", "v": 1}
        if tok in ("false", "False"):
            return {"op": "lit", "type": "bool", "v": 0}
        if tok[0].isdigit():
            if tok.endswith("u"):
                return {"op": "lit", "type": "u64", "v": int(tok[:-1], 0) & 0xFFFFFFFFFFFFFFFF}
            return {"op": "lit", "type": "i64", "v": int(tok, 0)}
        if tok in ("axis_var", "axis"):
            return {"op": "axis", "id": _hex(self._int_arg()), "type": "i64"}
        if tok in ("symbol_u64", "symbol"):
            return {"op": "sym", "id": _hex(self._int_arg())}
        if tok in ("task_tag_u64", "tag"):
            return {"op": "tag", "id": _hex(self._int_arg())}
        if tok in ("slot_u64", "slot_i64", "slot_bool"):
            return {"op": "slot", "i": self._int_arg(), "type": tok.split("_")[1]}
        if tok == "task_param":
            return {"op": "task_param", "i": self._int_arg()}
        if tok == "task":
            self.take(".")
            self.take("params")
            self.take("[")
            i = int(self.take(), 0)
            self.take("]")
            return {"op": "task_param", "i": i}
        raise ValueError(f"unsupported scalar expr token {tok!r} in {self.text!r}")


def parse_scalar_expr(text: str) -> dict:
    """Parse a printed ScalarExpr (C++ ``print`` or Python debug form)."""
    return _ExprParser(text).parse()


# ---------------------------------------------------------------------------
# ir::Module -> plan
# ---------------------------------------------------------------------------


def _axis_arg(a: Any) -> dict:
    # CodegenAxisArg (codegen.hpp:28-32); encoding as axis_arg_to_u64_literal
    # (pto_codegen.cpp:188-198).
    if a.is_var:
        return {"var": str(a.var)}
    if a.var:
        return {"sym": _hex(a.u64)}
    return {"u64": _hex(a.u64)}


def _tensor_arg(t: Any) -> dict:
    idx = []
    for e in t.index_exprs:
        idx.append({"var": str(e.var)} if e.is_var else {"const": int(e.constant)})
    return {
        "param": str(t.param),
        "tensor": int(t.tensor_id),
        "base_rank": int(t.base_rank),
        "view_rank": int(t.view_rank),
        "index": idx,
    }


def _axis(ax: Any, cpp: Any) -> dict:
    if isinstance(ax, cpp.DenseAxisNode):
        return {"kind": "dense", "size": int(ax.size)}
    if isinstance(ax, cpp.DenseDynAxisNode):
        return {"kind": "dense_dyn"}
    if isinstance(ax, cpp.RaggedAxisNode):
        return {
            "kind": "ragged",
            "outer_sym": _hex(fnv1a_64(str(ax.outer_size_var))),
            "lengths_sym": _hex(fnv1a_64(str(ax.lengths_var))),
        }
    raise ValueError(f"unsupported axis node {type(ax).__name__}")


def _node(n: Any, cpp: Any) -> dict:
    if isinstance(n, cpp.ParallelForNode) or isinstance(n, cpp.ForEachNode):
        kind = "parallel_for" if isinstance(n, cpp.ParallelForNode) else "for_each"
        return {"kind": kind, "var": str(n.index_var), "axis": _axis(n.axis, cpp), "body": _node(n.body, cpp)}
    if isinstance(n, cpp.TaskNode):
        return {
            "kind": "task",
            "kernel": str(n.kernel_name),
            "axis_args": [_axis_arg(a) for a in n.axis_args],
            "scalar_args": [_axis_arg(a) for a in n.scalar_args],
            "tensor_args": [_tensor_arg(t) for t in n.tensor_args],
        }
    if isinstance(n, cpp.CombineNode):
        return {"kind": "combine", "children": [_node(c, cpp) for c in n.workloads]}
    if isinstance(n, cpp.SequentialNode):
        return {"kind": "sequential", "children": [_node(c, cpp) for c in n.workloads]}
    if isinstance(n, cpp.CondNode):
        return {
            "kind": "cond",
            "pred": parse_scalar_expr(n.predicate.print()),
            "then": _node(n.then_branch, cpp),
            "else": _node(n.else_branch, cpp),
        }
    if isinstance(n, cpp.SelectNode):
        sp = n.sparse
        return {
            "kind": "select",
            "var": str(n.index_var),
            "outer_sym": _hex(fnv1a_64(str(sp.outer_size_var))),
            "indptr_sym": _hex(fnv1a_64(str(sp.indptr_var))),
            "indices_sym": _hex(fnv1a_64(str(sp.indices_var))),
            "body": _node(n.body, cpp),
        }
    if isinstance(n, cpp.SlotSetU64Node):
        return {"kind": "slot_set", "slot": int(n.slot), "value": _hex(n.value)}
    if isinstance(n, cpp.SlotLoadU64Node):
        return {"kind": "slot_load", "slot": int(n.slot), "tensor_arg": _tensor_arg(n.tensor),
                "row": int(n.row), "col": int(n.col)}
    if isinstance(n, cpp.PipelineNode):
        return {
            "kind": "pipeline",
            "channels": [{"name": str(c.name), "capacity": int(c.type.capacity)} for c in n.channels],
            "processes": [{"name": str(p.name), "produces": [str(x) for x in p.produces],
                           "consumes": [str(x) for x in p.consumes], "body": _node(p.body, cpp)}
                          for p in n.processes],
        }
    if isinstance(n, cpp.SendNode):
        return {"kind": "send", "channel": str(n.channel_name), "value": _node(n.value, cpp)}
    if isinstance(n, cpp.ConsumeNode):
        return {"kind": "consume", "channel": str(n.channel_name), "var": str(n.value_var), "body": _node(n.body, cpp)}
    raise ValueError(f"workload node {type(n).__name__} is not supported by the cuda_sm100a target")


def _attr_value(v: Any) -> Any:
    if isinstance(v, (bool, int, float, str)):
        return v
    if isinstance(v, (list, tuple)):
        return [_attr_value(x) for x in v]
    raise ValueError(f"unsupported attr value {v!r}")


def _kernel(kd: Any) -> dict:
    values = []
    for vid, vi in sorted(kd.values.items()):
        rows, cols = (int(vi.rows), int(vi.cols)) if vi.has_shape else (-1, -1)
        values.append([int(vid), _dtype(vi.dtype), rows, cols])
    ops = []
    for o in kd.ops:
        ops.append({
            "kind": str(o.kind),
            "result": int(o.result) if o.has_result else -1,
            "operands": [int(x) for x in o.operands],
            "attrs": {str(k): _attr_value(v) for k, v in dict(o.attrs).items()},
        })
    return {
        "name": str(kd.name),
        "params": [{"name": str(p.name), "id": int(p.id)} for p in kd.params],
        "values": values,
        "ops": ops,
        "attrs": {str(k): _attr_value(v) for k, v in dict(kd.attrs).items()},
    }


_POLICIES = {"RoundRobin": "round_robin", "Affinity": "affinity", "Hash": "hash",
             "WorkSteal": "work_steal", "Custom": "custom"}


def _schedule(module: Any, cpp: Any) -> dict:
    # Mirrors the directive scan of emit_workload_cpp_from_ir_ast
    # (pto_codegen.cpp:1500-1560): first Dispatch, first TaskWindow, first Stream.
    out: dict[str, Any] = {"dispatch": None, "task_window": None, "streams": 0, "unsupported": []}
    wl = module.workloads[0]
    sched = None
    for s in module.schedules:
        if getattr(s, "workload_name", None) in (wl.name, None) or len(module.schedules) == 1:
            sched = s
            break
    if sched is None:
        return out
    for d in sched.directives:
        if isinstance(d, cpp.DispatchNode):
            if out["dispatch"] is None:
                pol = _POLICIES.get(str(d.policy).split(".")[-1], "round_robin")
                key = None
                ktxt = str(d.key_expr or "")
                if pol in ("affinity", "hash", "custom") and ktxt:
                    key = parse_scalar_expr(ktxt)
                out["dispatch"] = {"policy": pol, "num_targets": int(d.num_targets), "key": key}
        elif isinstance(d, cpp.TaskWindowNode):
            if out["task_window"] is None:
                ov = str(d.overflow).split(".")[-1].lower()
                out["task_window"] = {"size": int(d.size), "unit": str(d.unit), "overflow": ov}
        elif isinstance(d, cpp.StreamNode):
            if not out["streams"]:
                out["streams"] = int(d.num_streams)
        else:
            out["unsupported"].append(type(d).__name__)
    return out


def module_to_plan(module: Any, cpp: Any = None) -> dict:
    """Serialise a reference ``ir::Module`` (pybind) into a plan dict."""
    if cpp is None:
        import importlib

        cpp = importlib.import_module(type(module).__module__)
    if not module.workloads:
        raise ValueError("Module has no workloads")
    wl = module.workloads[0]
    return {
        "format": PLAN_FORMAT,
        "name": str(module.name) if module.name else "main",
        "tensors": [{"dtype": _dtype(t.dtype), "shape": [int(d) for d in t.shape]} for t in module.tensors],
        "kernels": [_kernel(k) for k in module.kernels],
        "body": _node(wl.body, cpp),
        "schedule": _schedule(module, cpp),
    }


def dumps(plan: dict) -> str:
    return json.dumps(plan, sort_keys=True, separators=(",", ":"))


def loads(text: str) -> dict:
    plan = json.loads(text)
    if plan.get("format") != PLAN_FORMAT:
        raise ValueError(f"not a {PLAN_FORMAT} plan")
    return plan


def kernel_by_name(plan: dict, name: str) -> dict:
    for k in plan["kernels"]:
        if k["name"] == name:
            return k
    raise KeyError(f"Missing kernel def for task: {name}")
