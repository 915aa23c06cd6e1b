"""Plans for generic kernels cut at their contractions into stages (matmul kernels + fused row programs)."""

import struct

import numpy as np

from pto_wsp_b200.workloads import KernelBuilder, _pfor, _plan, _schedule, _targ, _task


def f32_bits(x: float) -> str:
    return hex(struct.unpack("<I", struct.pack("<f", x))[0])


def attention_plan(batch, heads, q_tiles, kv_len, d=128, scale=0.088):
    """Per (b, h, q tile): out = softmax(scale * Q . K^T) . V with a 128-row f16 Q tile, an f16 K^T tile
    [d, kv_len] and an f32 V tile [kv_len, d] -- the reference attention example's kernel at full tile sizes (the
    first contraction f16 x f16 on tcgen05, the second f32 x f32 on CUDA cores).  Tensors: 0 = Q [B, H, QT, 128, d]
    f16, 1 = K^T [B, H, d, kv_len] f16, 2 = V [B, H, kv_len, d] f32, 3 = O [B, H, QT, 128, d] f32."""
    kb = KernelBuilder("attention_tile")
    q = kb.param("q", "f16", 128, d)
    kt = kb.param("k_t", "f16", d, kv_len)
    v = kb.param("v", "f32", kv_len, d)
    out = kb.param("out", "f32", 128, d)
    sc = kb.param("scale", "f32")
    s = kb.op("Matmul", [q, kt], ("f32", 128, kv_len))
    s = kb.op("Mul", [s, sc], ("f32", 128, kv_len))
    mx = kb.op("RowMax", [s], ("f32", 128, 1))
    s = kb.op("Sub", [s, mx], ("f32", 128, kv_len))
    e = kb.op("Exp", [s], ("f32", 128, kv_len))
    sm = kb.op("RowSum", [e], ("f32", 128, 1))
    w = kb.op("Div", [e, sm], ("f32", 128, kv_len))
    kb.store(out, kb.op("Matmul", [w, v], ("f32", 128, d)))
    body = _pfor("b", batch, _pfor("h", heads, _pfor("s", q_tiles, _task("attention_tile", ["b", "h", "s"], [
        _targ("q", 0, 5, ["b", "h", "s"]), _targ("k_t", 1, 4, ["b", "h"]), _targ("v", 2, 4, ["b", "h"]),
        _targ("out", 3, 5, ["b", "h", "s"])], [{"u64": f32_bits(scale)}]))))
    tensors = [("f16", [batch, heads, q_tiles, 128, d]), ("f16", [batch, heads, d, kv_len]),
               ("f32", [batch, heads, kv_len, d]), ("f32", [batch, heads, q_tiles, 128, d])]
    return _plan("attention", tensors, [kb.build()], body, _schedule())


def attention_arrays(rng, batch, heads, q_tiles, kv_len, d=128):
    q = rng.standard_normal((batch, heads, q_tiles, 128, d)).astype(np.float16)
    kt = rng.standard_normal((batch, heads, d, kv_len)).astype(np.float16)
    v = rng.standard_normal((batch, heads, kv_len, d)).astype(np.float32)
    o = np.full((batch, heads, q_tiles, 128, d), np.nan, np.float32)
    return [q, kt, v, o]


def mlp_plan(tiles, rows, d, hidden):
    """Per tile: out = x + relu(x . W1) . W2, all f32 (the reference llama example's MLP block with a residual) at
    tile sizes whose operands exceed shared memory.  Tensors: 0 = X [T, rows, d], 1 = W1 [d, hidden],
    2 = W2 [hidden, d], 3 = O [T, rows, d]."""
    kb = KernelBuilder("mlp_tile")
    x = kb.param("x", "f32", rows, d)
    w1 = kb.param("w1", "f32", d, hidden)
    w2 = kb.param("w2", "f32", hidden, d)
    out = kb.param("out", "f32", rows, d)
    h = kb.op("Matmul", [x, w1], ("f32", rows, hidden))
    z = kb.op("Constant", [], ("f32", -1, -1), value=0.0)
    r = kb.op("Max", [h, z], ("f32", rows, hidden))
    y = kb.op("Matmul", [r, w2], ("f32", rows, d))
    kb.store(out, kb.op("Add", [x, y], ("f32", rows, d)))
    body = _pfor("t", tiles, _task("mlp_tile", ["t"], [
        _targ("x", 0, 3, ["t"]), _targ("w1", 1, 2, []), _targ("w2", 2, 2, []), _targ("out", 3, 3, ["t"])]))
    tensors = [("f32", [tiles, rows, d]), ("f32", [d, hidden]), ("f32", [hidden, d]), ("f32", [tiles, rows, d])]
    return _plan("mlp", tensors, [kb.build()], body, _schedule())


def mlp_arrays(rng, tiles, rows, d, hidden):
    x = rng.standard_normal((tiles, rows, d)).astype(np.float32)
    w1 = (rng.standard_normal((d, hidden)) / np.sqrt(d)).astype(np.float32)
    w2 = (rng.standard_normal((hidden, d)) / np.sqrt(hidden)).astype(np.float32)
    return [x, w1, w2, np.full((tiles, rows, d), np.nan, np.float32)]


def inout_plan(tiles, n=128):
    """Per tile: p <- 2 p, then q = A . B + (p as it was): a param stored before a later stage needs its old value,
    which must come from scratch, not from the param.  Tensors: 0 = P, 1 = A, 2 = B, 3 = Q, all [T, n, n] f32."""
    kb = KernelBuilder("inout_tile")
    p = kb.param("p", "f32", n, n)
    a = kb.param("a", "f32", n, n)
    b = kb.param("b", "f32", n, n)
    q = kb.param("q", "f32", n, n)
    two = kb.op("Constant", [], ("f32", -1, -1), value=2.0)
    kb.store(p, kb.op("Mul", [p, two], ("f32", n, n)))
    m = kb.op("Matmul", [a, b], ("f32", n, n))
    kb.store(q, kb.op("Add", [m, p], ("f32", n, n)))
    body = _pfor("t", tiles, _task("inout_tile", ["t"], [
        _targ("p", 0, 3, ["t"]), _targ("a", 1, 3, ["t"]), _targ("b", 2, 3, ["t"]), _targ("q", 3, 3, ["t"])]))
    tensors = [("f32", [tiles, n, n])] * 4
    return _plan("inout", tensors, [kb.build()], body, _schedule())
