"""Plans for generic kernels that contract first and finish row-locally (a tcgen05 matmul + a fused row program)."""

import struct

import numpy as np

from pto_wsp_b200.workloads import KernelBuilder, _pfor, _plan, _schedule, _targ, _task


def f32_bits(x: float) -> str:
    return hex(struct.unpack("<I", struct.pack("<f", x))[0])


def mm_epilogue_plan(batch, m, n, k, tn=256, scale=0.125, bias_op="Sub"):
    """out = exp(s - rowmax(s)) with s = (A . B - bias) * scale per 128 x tn output tile; bias is a one-row [1, tn]
    operand (a column broadcast: tn != 128, else the emitter's row-broadcast rule takes a [1, 128] operand), scale
    a scalar param.  With tn = 128 and bias_op "Add" the bias is a row broadcast instead (element r to row r).  Tensors as in the bgemm plan: 0 = A [B, M/128, 128, K] f16,
    1 = B viewed [B, N/tn, K, tn] f16, 2 = bias [B, N/tn, 1, tn] f32, 3 = out viewed [B, M/128, N/tn, 128, tn] f32."""
    kb = KernelBuilder("mm_softmax_tile")
    a = kb.param("a", "f16", 128, k)
    b = kb.param("b", "f16", k, tn)
    bias = kb.param("bias", "f32", 1, tn)
    out = kb.param("out", "f32", 128, tn)
    sc = kb.param("scale", "f32")
    c = kb.op("Matmul", [a, b], ("f32", 128, tn))
    d = kb.op(bias_op, [c, bias], ("f32", 128, tn))
    e = kb.op("Mul", [d, sc], ("f32", 128, tn))
    mx = kb.op("RowMax", [e], ("f32", 128, 1))
    f = kb.op("Sub", [e, mx], ("f32", 128, tn))
    kb.store(out, kb.op("Exp", [f], ("f32", 128, tn)))
    body = _pfor("b", batch, _pfor("i", m // 128, _pfor("j", n // tn, _task("mm_softmax_tile", ["b", "i", "j"], [
        _targ("a", 0, 4, ["b", "i"]), _targ("b", 1, 4, ["b", "j"]), _targ("bias", 2, 4, ["b", "j"]),
        _targ("out", 3, 5, ["b", "i", "j"])], [{"u64": f32_bits(scale)}]))))
    tensors = [("f16", [batch, m // 128, 128, k]), ("f16", [batch, n // tn, k, tn]), ("f32", [batch, n // tn, 1, tn]),
               ("f32", [batch, m // 128, n // tn, 128, tn])]
    return _plan("mm_softmax", tensors, [kb.build()], body, _schedule())


def mm_epilogue_arrays(rng, batch, m, n, k, tn=256):
    A = rng.uniform(-1, 1, (batch, m, k)).astype(np.float16)
    Bf = rng.uniform(-1, 1, (batch, k, n)).astype(np.float16)
    bias = rng.standard_normal((batch, n)).astype(np.float32)
    C = np.full((batch, m, n), np.nan, np.float32)
    a = A.reshape(batch, m // 128, 128, k)
    b = Bf.reshape(batch, k, n // tn, tn).transpose(0, 2, 1, 3)
    bs = bias.reshape(batch, n // tn, 1, tn)
    c = C.reshape(batch, m // 128, 128, n // tn, tn).transpose(0, 1, 3, 2, 4)
    return (A, Bf, bias, C), [a, b, bs, c]
