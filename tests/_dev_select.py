"""A plan whose `P.when` tiers over a slot loaded from a tensor pick a task's scalar (device-selected scalars)."""

import struct

from pto_wsp_b200.workloads import KernelBuilder, _pfor, _plan, _schedule, _targ


def _f32(x):
    return hex(struct.unpack("<I", struct.pack("<f", x))[0])


def _task(scale):
    return {"kind": "task", "kernel": "scale_tile", "axis_args": [{"var": "b"}, {"var": "t"}],
            "scalar_args": [{"u64": _f32(scale)}],
            "tensor_args": [_targ("x", 1, 4, ["b", "t"]), _targ("out", 2, 4, ["b", "t"])]}


def _cmp(fn, lit, slot_type):
    return {"op": "bin", "fn": fn, "a": {"op": "slot", "i": 0, "type": slot_type}, "b": {"op": "lit", "type": "i64", "v": lit}}


def tiered_scale_plan(B, T, R=8, C=64, src_dtype="i32", slot_type="i64", tiers=((-5, 0.5), (10, 1.0), (100, 2.0)),
                      last=3.0):
    """out[b][t] = x[b][t] * s, s by the first tier with sel[b][t] <= bound, else `last`; sel is [B, T, 1, 1]."""
    k = KernelBuilder("scale_tile")
    x = k.param("x", "f32", R, C)
    out = k.param("out", "f32", R, C)
    s = k.param("s", "f32")
    k.store(out, k.op("Mul", [x, s], ("f32", R, C)))
    tree = _task(last)
    for bound, scale in reversed(tiers):
        tree = {"kind": "cond", "pred": _cmp("<=", bound, slot_type), "then": _task(scale), "else": tree}
    load = {"kind": "slot_load", "slot": 0, "tensor_arg": _targ("sel", 0, 4, ["b", "t"]), "row": 0, "col": 0}
    body = _pfor("b", B, _pfor("t", T, {"kind": "sequential", "children": [load, tree]}))
    return _plan("tiered_scale", [(src_dtype, [B, T, 1, 1]), ("f32", [B, T, R, C]), ("f32", [B, T, R, C])],
                 [k.build()], body, _schedule())


def expected_scale(v, tiers=((-5, 0.5), (10, 1.0), (100, 2.0)), last=3.0):
    for bound, scale in tiers:
        if v <= bound:
            return scale
    return last
