"""The five BASELINE workloads as plans, at any size.

Each builder returns the plan the reference frontend produces for the same
``@kernel`` / ``@workload`` code (``tests/test_workload_plans.py`` checks this
against ``workload_to_codegen_ir`` + :func:`pto_wsp_b200.plan.module_to_plan`),
so the GPU box can run the exact workloads without the reference installed.
The matching frontend code is given in each docstring.

Shapes follow BASELINE.json:

1. RMSNorm tiles      X[B,T,16,128] f32, ``x * rsqrt(rowmean(x*x))``
2. row softmax tiles  X[B,T,32,256] f32, ``exp(x - rowmax) / rowsum``
3. bgemm              C[b] = A[b] @ B[b], 128x128 output tiles, K inside the kernel
4. paged GQA decode   built-in custom kernel over a paged KV cache
5. lightning indexer  built-in scoring + built-in top-k
"""

from __future__ import annotations

from typing import Any

from .plan import PLAN_FORMAT

_VAR_NAMES = ["b", "h", "s", "d", "i", "j", "k", "l", "m", "n"]


def _schedule(num_aicpus: int = 4, window: int = 8192, policy: str = "round_robin", key: dict | None = None) -> dict:
    return {
        "dispatch": {"policy": policy, "num_targets": num_aicpus, "key": key},
        "task_window": {"size": window, "unit": "tasks", "overflow": "stall"},
        "streams": 0,
        "unsupported": [],
    }


class KernelBuilder:
    """Builds a ``CodegenKernelDef`` the way the reference tracer numbers values."""

    def __init__(self, name: str):
        self.name = name
        self.params: list[dict] = []
        self.values: list[list] = []
        self.ops: list[dict] = []
        self.attrs: dict[str, Any] = {}
        self._next = 1

    def param(self, name: str, dtype: str, rows: int = -1, cols: int = -1) -> int:
        vid = self._next
        self._next += 1
        self.params.append({"name": name, "id": vid})
        self.values.append([vid, dtype, rows, cols])
        return vid

    def op(self, kind: str, operands: list[int], result: tuple[str, int, int] | None = None, **attrs) -> int:
        rid = -1
        if result is not None:
            rid = self._next
            self._next += 1
            self.values.append([rid, result[0], result[1], result[2]])
        self.ops.append({"kind": kind, "result": rid, "operands": list(operands), "attrs": dict(attrs)})
        return rid

    def store(self, dst: int, src: int) -> None:
        self.op("Store", [dst, src], None, offset=[0, 0])

    def build(self) -> dict:
        return {"name": self.name, "params": self.params, "values": sorted(self.values), "ops": self.ops,
                "attrs": self.attrs}


def _task(kernel: str, axis_vars: list[str], tensor_args: list[dict], scalar_args: list[dict] | None = None) -> dict:
    return {"kind": "task", "kernel": kernel, "axis_args": [{"var": v} for v in axis_vars],
            "scalar_args": scalar_args or [], "tensor_args": tensor_args}


def _targ(param: str, tensor: int, base_rank: int, index: list) -> dict:
    idx = [{"var": i} if isinstance(i, str) else {"const": int(i)} for i in index]
    return {"param": param, "tensor": tensor, "base_rank": base_rank, "view_rank": base_rank - len(idx), "index": idx}


def _pfor(var: str, size: int | None, body: dict, seq: bool = False) -> dict:
    axis = {"kind": "dense", "size": int(size)} if size is not None else {"kind": "dense_dyn"}
    return {"kind": "for_each" if seq else "parallel_for", "var": var, "axis": axis, "body": body}


def _plan(name: str, tensors: list[tuple[str, list[int]]], kernels: list[dict], body: dict, schedule: dict) -> dict:
    return {"format": PLAN_FORMAT, "name": name,
            "tensors": [{"dtype": dt, "shape": [int(x) for x in shp]} for dt, shp in tensors],
            "kernels": kernels, "body": body, "schedule": schedule}


# ---------------------------------------------------------------------------
# 1. RMSNorm
# ---------------------------------------------------------------------------


def rmsnorm_plan(batch: int, tiles: int, rows: int = 16, cols: int = 128, name: str = "rmsnorm") -> dict:
    """Frontend form (``examples/e2e_rmsnorm/pto_wsp_impl.py:43-68``)::

        @kernel
        def rmsnorm_tile(x: In[Tile[16,128,F32]], out: Out[Tile[16,128,F32]]):
            sq = pto.mul(x, x); mean_sq = pto.rowmean(sq); inv = pto.rsqrt(mean_sq)
            pto.store(out, pto.mul(x, inv))
        for b in P(Dense[B]()):
            for t in P(Dense[T]()):
                rmsnorm_tile[b, t](x=X[b][t], out=Y[b][t])
        .dispatch(DispatchPolicy.round_robin(num_aicpus=4)).task_graph(window=TaskWindow(8192, "tasks", STALL))

    Tensors: 0 = X [B,T,rows,cols] f32, 1 = Y [B,T,rows,cols] f32.
    """
    k = KernelBuilder("rmsnorm_tile")
    x = k.param("x", "f32", rows, cols)
    out = k.param("out", "f32", rows, cols)
    sq = k.op("Mul", [x, x], ("f32", rows, cols))
    mean = k.op("RowMean", [sq], ("f32", rows, 1))
    inv = k.op("Rsqrt", [mean], ("f32", rows, 1))
    y = k.op("Mul", [x, inv], ("f32", rows, cols))
    k.store(out, y)
    b, t = _VAR_NAMES[0], _VAR_NAMES[1]
    body = _pfor(b, batch, _pfor(t, tiles, _task("rmsnorm_tile", [b, t], [
        _targ("x", 0, 4, [b, t]), _targ("out", 1, 4, [b, t])])))
    return _plan(name, [("f32", [batch, tiles, rows, cols]), ("f32", [batch, tiles, rows, cols])], [k.build()], body,
                 _schedule())


# ---------------------------------------------------------------------------
# 2. Row softmax
# ---------------------------------------------------------------------------


def softmax_plan(batch: int, tiles: int, rows: int = 32, cols: int = 256, name: str = "softmax") -> dict:
    """Frontend form::

        @kernel
        def softmax_tile(x: In[Tile[32,256,F32]], out: Out[Tile[32,256,F32]]):
            m = pto.rowmax(x); e = pto.exp(pto.sub(x, m)); s = pto.rowsum(e)
            pto.store(out, pto.div(e, s))
        for b in P(Dense[B]()):
            for t in P(Dense[T]()):
                softmax_tile[b, t](x=X[b][t], out=Y[b][t])

    Tensors: 0 = X [B,T,rows,cols] f32, 1 = Y [B,T,rows,cols] f32.
    """
    k = KernelBuilder("softmax_tile")
    x = k.param("x", "f32", rows, cols)
    out = k.param("out", "f32", rows, cols)
    m = k.op("RowMax", [x], ("f32", rows, 1))
    d = k.op("Sub", [x, m], ("f32", rows, cols))
    e = k.op("Exp", [d], ("f32", rows, cols))
    s = k.op("RowSum", [e], ("f32", rows, 1))
    y = k.op("Div", [e, s], ("f32", rows, cols))
    k.store(out, y)
    b, t = _VAR_NAMES[0], _VAR_NAMES[1]
    body = _pfor(b, batch, _pfor(t, tiles, _task("softmax_tile", [b, t], [
        _targ("x", 0, 4, [b, t]), _targ("out", 1, 4, [b, t])])))
    return _plan(name, [("f32", [batch, tiles, rows, cols]), ("f32", [batch, tiles, rows, cols])], [k.build()], body,
                 _schedule())


# ---------------------------------------------------------------------------
# 3. bgemm
# ---------------------------------------------------------------------------


def bgemm_plan(batch: int, m: int, n: int, k: int, tile_m: int = 128, tile_n: int = 128, accumulate: bool = False,
               name: str = "bgemm") -> dict:
    """Frontend form (K loop inside the kernel; cf. ``examples/bgemm/pto_wsp_impl.py:56-76``)::

        @kernel
        def gemm_tile(a: In[Tile[128,K,F16]], b: In[Tile[K,128,F16]], c: Out[Tile[128,128,F32]]):
            pto.store(c, pto.matmul(a, b))          # accumulate=True: pto.store(c, pto.add(c, pto.matmul(a, b)))
        for b in P(Dense[B]()):
            for tm in P(Dense[M/128]()):
                for tn in P(Dense[N/128]()):
                    gemm_tile[b, tm, tn](a=A[b][tm], b=Bt[b][tn], c=C[b][tm][tn])

    Tensors (numpy views of contiguous A[B,M,K], B[B,K,N], C[B,M,N]):
      0 = A.reshape(B, M/tm, tm, K)                                   f16
      1 = B.reshape(B, K, N/tn, tn).transpose(0, 2, 1, 3)  [B,N/tn,K,tn] f16
      2 = C.reshape(B, M/tm, tm, N/tn, tn).transpose(0,1,3,2,4) [B,M/tm,N/tn,tm,tn] f32
    """
    kb = KernelBuilder("gemm_tile")
    a = kb.param("a", "f16", tile_m, k)
    bb = kb.param("b", "f16", k, tile_n)
    c = kb.param("c", "f32", tile_m, tile_n)
    acc = kb.op("Matmul", [a, bb], ("f32", tile_m, tile_n))
    if accumulate:
        acc = kb.op("Add", [c, acc], ("f32", tile_m, tile_n))
    kb.store(c, acc)
    v0, v1, v2 = _VAR_NAMES[:3]
    body = _pfor(v0, batch, _pfor(v1, m // tile_m, _pfor(v2, n // tile_n, _task("gemm_tile", [v0, v1, v2], [
        _targ("a", 0, 4, [v0, v1]), _targ("b", 1, 4, [v0, v2]), _targ("c", 2, 5, [v0, v1, v2])]))))
    tensors = [("f16", [batch, m // tile_m, tile_m, k]), ("f16", [batch, n // tile_n, k, tile_n]),
               ("f32", [batch, m // tile_m, n // tile_n, tile_m, tile_n])]
    return _plan(name, tensors, [kb.build()], body, _schedule())


# ---------------------------------------------------------------------------
# 4. Paged GQA decode (built-in custom kernel)
# ---------------------------------------------------------------------------

PAGED_DECODE_CPU_BODY = r"""// ptowsp-builtin: paged_decode_gqa
// Reference CPU-sim body (plain C++): one (request, kv_head) task of paged GQA decode.
// q[G,D] f16 | k_cache, v_cache f16 paged [pages, page_size, KVH, D] (s3 = page, s4 = token stride)
// page_table[1, maxp] i32 | kv_len[1,1] i32 | out[G,D] f16 | axis args (r, h) | scalars page_size, KVH
const int nt = 6;
const uint32_t tail = task->num_axis_args - 2 * nt;
const int G = (int)task->args[tail + 0], D = (int)task->args[tail + 1];
const int h = (int)task->args[1];
const int page_size = (int)task->args[task->num_axis_args + 0];
const _Float16* q = (const _Float16*)task->tensor_ptrs[0];
const _Float16* kc = (const _Float16*)task->tensor_ptrs[1];
const _Float16* vc = (const _Float16*)task->tensor_ptrs[2];
const int32_t* pt = (const int32_t*)task->tensor_ptrs[3];
const int32_t L = *(const int32_t*)task->tensor_ptrs[4];
_Float16* out = (_Float16*)task->tensor_ptrs[5];
const uint64_t q_s3 = task->tensor_strides[0], k_s3 = task->tensor_strides[2], k_s4 = task->tensor_strides[3];
const uint64_t v_s3 = task->tensor_strides[4], v_s4 = task->tensor_strides[5], pt_s4 = task->tensor_strides[7];
const uint64_t o_s3 = task->tensor_strides[10];
const float scale = 1.0f / __builtin_sqrtf((float)D);
for (int g = 0; g < G; ++g) {
  float m = -__builtin_inff(), l = 0.f, acc[256] = {0};
  for (int t = 0; t < L; ++t) {
    const int64_t page = pt[(t / page_size) * pt_s4];
    const _Float16* kr = kc + page * k_s3 + (t % page_size) * k_s4 + h * D;
    const _Float16* vr = vc + page * v_s3 + (t % page_size) * v_s4 + h * D;
    float s = 0.f;
    for (int d = 0; d < D; ++d) s += (float)q[g * q_s3 + d] * (float)kr[d];
    s *= scale;
    const float mn = s > m ? s : m, c = __builtin_expf(m - mn), p = __builtin_expf(s - mn);
    l = l * c + p;
    for (int d = 0; d < D; ++d) acc[d] = acc[d] * c + p * (float)vr[d];
    m = mn;
  }
  for (int d = 0; d < D; ++d) out[g * o_s3 + d] = (_Float16)(L > 0 ? acc[d] / l : 0.f);
}
"""


def decode_plan(requests: int, kv_heads: int, group: int, head_dim: int, num_pages: int, max_pages: int,
                page_size: int = 16, name: str = "paged_decode") -> dict:
    """Frontend form::

        @kernel(cpp_src=PAGED_DECODE_CPU_BODY)
        def paged_decode(q: In[Tile[G,D,F16]], k_cache: In[Tile[page_size,KVH*D,F16]],
                         v_cache: In[Tile[page_size,KVH*D,F16]], page_table: In[Tile[1,maxp,I32]],
                         kv_len: In[Tile[1,1,I32]], out: Out[Tile[G,D,F16]],
                         page_size: Scalar[I32] = 16, num_kv_heads: Scalar[I32] = KVH): ...
        for b in P(DenseDyn(R)):
            for h in P(Dense[KVH]()):
                paged_decode[b, h](q=Q[b][h], k_cache=KC, v_cache=VC, page_table=PT[b], kv_len=KL[b], out=O[b][h])

    Tensors: 0 = Q [R,KVH,G,D] f16, 1 = KC [pages,page_size,KVH,D] f16, 2 = VC (same), 3 = PT [R,maxp] i32,
    4 = KL [R,1] i32, 5 = O [R,KVH,G,D] f16.  The request axis is DenseDyn (axis size "b").
    """
    kb = KernelBuilder("paged_decode")
    kb.param("q", "f16", group, head_dim)
    kb.param("k_cache", "f16", page_size, kv_heads * head_dim)
    kb.param("v_cache", "f16", page_size, kv_heads * head_dim)
    kb.param("page_table", "i32", 1, max_pages)
    kb.param("kv_len", "i32", 1, 1)
    kb.param("out", "f16", group, head_dim)
    kb.param("page_size", "i32")
    kb.param("num_kv_heads", "i32")
    kb.attrs = {"cpp_src": PAGED_DECODE_CPU_BODY}
    b, h = _VAR_NAMES[:2]
    body = _pfor(b, None, _pfor(h, kv_heads, _task("paged_decode", [b, h], [
        _targ("q", 0, 4, [b, h]), _targ("k_cache", 1, 4, []), _targ("v_cache", 2, 4, []),
        _targ("page_table", 3, 2, [b]), _targ("kv_len", 4, 2, [b]), _targ("out", 5, 4, [b, h])],
        [{"u64": hex(page_size)}, {"u64": hex(kv_heads)}])))
    tensors = [("f16", [requests, kv_heads, group, head_dim]), ("f16", [num_pages, page_size, kv_heads, head_dim]),
               ("f16", [num_pages, page_size, kv_heads, head_dim]), ("i32", [requests, max_pages]),
               ("i32", [requests, 1]), ("f16", [requests, kv_heads, group, head_dim])]
    return _plan(name, tensors, [kb.build()], body, _schedule())


# ---------------------------------------------------------------------------
# 5. Lightning indexer + top-k (built-in custom kernels)
# ---------------------------------------------------------------------------

INDEXER_SCORE_CPU_BODY = r"""// ptowsp-builtin: lightning_indexer_score
// Reference CPU-sim body (plain C++): scores[q,t] = sum_h w[q,h] * relu(q[q*H+h,:] . k[t,:]).
const int nt = 4;
const uint32_t tail = task->num_axis_args - 2 * nt;
const int QH = (int)task->args[tail + 0], D = (int)task->args[tail + 1];
const int T = (int)task->args[tail + 2];
const int Q = (int)task->args[tail + 4], H = (int)task->args[tail + 5];
const _Float16* q = (const _Float16*)task->tensor_ptrs[0];
const _Float16* k = (const _Float16*)task->tensor_ptrs[1];
const float* w = (const float*)task->tensor_ptrs[2];
float* s = (float*)task->tensor_ptrs[3];
const uint64_t q_s3 = task->tensor_strides[0], k_s3 = task->tensor_strides[2];
const uint64_t w_s3 = task->tensor_strides[4], s_s3 = task->tensor_strides[6];
(void)QH;
for (int qi = 0; qi < Q; ++qi)
  for (int t = 0; t < T; ++t) {
    float acc = 0.f;
    for (int hh = 0; hh < H; ++hh) {
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot += (float)q[(qi * H + hh) * q_s3 + d] * (float)k[t * k_s3 + d];
      acc += w[qi * w_s3 + hh] * (dot > 0.f ? dot : 0.f);
    }
    s[qi * s_s3 + t] = acc;
  }
"""

TOPK_CPU_BODY = r"""// ptowsp-builtin: topk_select
// Reference CPU-sim body (plain C++): indices of the K largest scores, ties -> lower index
// (the TSORT32 rule of examples/deepseek_lightning_indexer/golden.py).
const int nt = 2;
const uint32_t tail = task->num_axis_args - 2 * nt;
const int N = (int)task->args[tail + 1], K = (int)task->args[tail + 3];
const float* s = (const float*)task->tensor_ptrs[0];
int32_t* out = (int32_t*)task->tensor_ptrs[1];
const uint64_t s_s4 = task->tensor_strides[1], o_s4 = task->tensor_strides[3];
for (int i = 0; i < K; ++i) out[i * o_s4] = -1;
for (int n = 0; n < N; ++n) {
  const float v = s[n * s_s4];
  int pos = K;
  while (pos > 0) {
    const int32_t j = out[(pos - 1) * o_s4];
    if (j >= 0 && !(v > s[j * s_s4])) break;
    if (pos < K) out[pos * o_s4] = j;
    --pos;
  }
  if (pos < K) out[pos * o_s4] = n;
}
"""


def indexer_plan(batch: int, queries: int, heads: int, head_dim: int, context: int, topk: int,
                 name: str = "lightning_indexer") -> dict:
    """Frontend form::

        @kernel(cpp_src=INDEXER_SCORE_CPU_BODY)
        def indexer_score(q: In[Tile[Q*H,D,F16]], k: In[Tile[T,D,F16]], w: In[Tile[Q,H,F32]],
                          scores: Out[Tile[Q,T,F32]]): ...
        @kernel(cpp_src=TOPK_CPU_BODY)
        def topk(scores: In[Tile[1,T,F32]], out: Out[Tile[1,K,I32]]): ...
        for b in P(Dense[B]()):
            indexer_score[b](q=Qt[b], k=Kt[b], w=W[b], scores=S[b])
        for b2 in P(Dense[B]()):
            for q in P(Dense[Q]()):
                topk[b2, q](scores=S[b2][q], out=I[b2][q])

    Tensors: 0 = Q [B,Q*H,D] f16, 1 = K [B,T,D] f16, 2 = W [B,Q,H] f32, 3 = S [B,Q,T] f32, 4 = I [B,Q,K] i32.
    """
    ks = KernelBuilder("indexer_score")
    ks.param("q", "f16", queries * heads, head_dim)
    ks.param("k", "f16", context, head_dim)
    ks.param("w", "f32", queries, heads)
    ks.param("scores", "f32", queries, context)
    ks.attrs = {"cpp_src": INDEXER_SCORE_CPU_BODY}
    kt = KernelBuilder("topk")
    kt.param("scores", "f32", 1, context)
    kt.param("out", "i32", 1, topk)
    kt.attrs = {"cpp_src": TOPK_CPU_BODY}
    v0, v1, v2 = _VAR_NAMES[:3]
    n1 = _pfor(v0, batch, _task("indexer_score", [v0], [
        _targ("q", 0, 3, [v0]), _targ("k", 1, 3, [v0]), _targ("w", 2, 3, [v0]), _targ("scores", 3, 3, [v0])]))
    n2 = _pfor(v1, batch, _pfor(v2, queries, _task("topk", [v1, v2], [
        _targ("scores", 3, 3, [v1, v2]), _targ("out", 4, 3, [v1, v2])])))
    tensors = [("f16", [batch, queries * heads, head_dim]), ("f16", [batch, context, head_dim]),
               ("f32", [batch, queries, heads]), ("f32", [batch, queries, context]), ("i32", [batch, queries, topk])]
    return _plan(name, [*tensors], [ks.build(), kt.build()], {"kind": "combine", "children": [n1, n2]}, _schedule())


# ---------------------------------------------------------------------------
# Attention tiles (the reference attention example's kernel at full tile sizes)
# ---------------------------------------------------------------------------


def attention_plan(batch: int, heads: int, q_tiles: int, kv_len: int, d: int = 128, scale: float | None = 0.088,
                   v_dtype: str = "f32", name: str = "attention") -> dict:
    """Frontend form (``examples/attention/pto_wsp_impl.py:51-68`` with f16 Q / K^T tiles)::

        @kernel
        def attention_tile(q: In[Tile[128, D, F16]], k_t: In[Tile[D, L, F16]], v: In[Tile[L, D, F32]],
                           out: Out[Tile[128, D, F32]], scale: Scalar[F32]):
            s = pto.mul(pto.matmul(q, k_t), scale)
            w = pto.div(pto.exp(pto.sub(s, pto.rowmax(s))), pto.rowsum(...))
            pto.store(out, pto.matmul(w, v))
        for b in P(Dense[B]()):
            for h in P(Dense[H]()):
                for s in P(Dense[QT]()):
                    attention_tile[b, h, s](q=Q[b][h][s], k_t=KT[b][h], v=V[b][h], out=O[b][h][s], scale=scale)

    The softmax result is f32 (pto has no cast), so V is f32 too: the emitter takes a matmul only with both
    operands f16 or both f32.  With d = 128 and L a multiple of 64 this is the fused tcgen05 attention kernel's
    pattern; ``scale=None`` leaves the multiply out.  Tensors: 0 = Q [B, H, QT, 128, d] f16, 1 = K^T [B, H, d, L]
    f16, 2 = V [B, H, L, d] f32, 3 = O [B, H, QT, 128, d] f32.
    """
    import struct

    kb = KernelBuilder("attention_tile")
    q = kb.param("q", "f16", 128, d)
    kt = kb.param("k_t", "f16", d, kv_len)
    v = kb.param("v", v_dtype, kv_len, d)
    out = kb.param("out", "f32", 128, d)
    scalars = []
    s = kb.op("Matmul", [q, kt], ("f32", 128, kv_len))
    if scale is not None:
        sc = kb.param("scale", "f32")
        s = kb.op("Mul", [s, sc], ("f32", 128, kv_len))
        scalars = [{"u64": hex(struct.unpack("<I", struct.pack("<f", scale))[0])}]
    mx = kb.op("RowMax", [s], ("f32", 128, 1))
    s = kb.op("Sub", [s, mx], ("f32", 128, kv_len))
    e = kb.op("Exp", [s], ("f32", 128, kv_len))
    sm = kb.op("RowSum", [e], ("f32", 128, 1))
    w = kb.op("Div", [e, sm], ("f32", 128, kv_len))
    kb.store(out, kb.op("Matmul", [w, v], ("f32", 128, d)))
    body = _pfor("b", batch, _pfor("h", heads, _pfor("s", q_tiles, _task("attention_tile", ["b", "h", "s"], [
        _targ("q", 0, 5, ["b", "h", "s"]), _targ("k_t", 1, 4, ["b", "h"]), _targ("v", 2, 4, ["b", "h"]),
        _targ("out", 3, 5, ["b", "h", "s"])], scalars))))
    tensors = [("f16", [batch, heads, q_tiles, 128, d]), ("f16", [batch, heads, d, kv_len]),
               (v_dtype, [batch, heads, kv_len, d]), ("f32", [batch, heads, q_tiles, 128, d])]
    return _plan(name, tensors, [kb.build()], body, _schedule())


def attention_inputs(rng, batch: int, heads: int, q_tiles: int, kv_len: int, d: int = 128, v_dtype: str = "f32"):
    """Q, K^T, V ~ N(0,1) (f16, V in `v_dtype`), O filled with NaN."""
    import numpy as np

    q = rng.standard_normal((batch, heads, q_tiles, 128, d), dtype=np.float32).astype(np.float16)
    kt = rng.standard_normal((batch, heads, d, kv_len), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((batch, heads, kv_len, d), dtype=np.float32).astype(
        np.float16 if v_dtype == "f16" else np.float32)
    o = np.full((batch, heads, q_tiles, 128, d), np.nan, np.float32)
    return [q, kt, v, o]


def bgemm_views(a, b, c, tile_m: int = 128, tile_n: int = 128):
    """The bgemm plan's tensor views of contiguous A[B,M,K], B[B,K,N], C[B,M,N] (numpy or torch)."""
    Bn, M, K = a.shape
    N = b.shape[2]
    av = a.reshape(Bn, M // tile_m, tile_m, K)
    if hasattr(b, "permute"):
        bv = b.reshape(Bn, K, N // tile_n, tile_n).permute(0, 2, 1, 3)
        cv = c.reshape(Bn, M // tile_m, tile_m, N // tile_n, tile_n).permute(0, 1, 3, 2, 4)
    else:
        bv = b.reshape(Bn, K, N // tile_n, tile_n).transpose(0, 2, 1, 3)
        cv = c.reshape(Bn, M // tile_m, tile_m, N // tile_n, tile_n).transpose(0, 1, 3, 2, 4)
    return av, bv, cv


def topk_plan(rows: int, n: int, k: int, name: str = "topk_rows") -> dict:
    """Top-k rows alone: ``for b in P(rows): topk[b](scores=S[b], out=I[b])`` (S [rows,1,n], I [rows,1,k])."""
    kt = KernelBuilder("topk")
    kt.param("scores", "f32", 1, n)
    kt.param("out", "i32", 1, k)
    kt.attrs = {"cpp_src": TOPK_CPU_BODY}
    v0 = _VAR_NAMES[0]
    body = _pfor(v0, rows, _task("topk", [v0], [_targ("scores", 0, 3, [v0]), _targ("out", 1, 3, [v0])]))
    return _plan(name, [("f32", [rows, 1, n]), ("i32", [rows, 1, k])], [kt.build()], body, _schedule())


# ---------------------------------------------------------------------------
# Seeded synthetic inputs (BASELINE.json distributions)
# ---------------------------------------------------------------------------


def decode_inputs(rng, requests: int, kv_heads: int = 8, group: int = 4, head_dim: int = 128, page_size: int = 16,
                  lengths=None, lo: int = 512, hi: int = 8192, max_pages: int | None = None):
    """Q/K/V ~ N(0,1) f16, KV lengths ~ U{lo..hi}, pages = one random permutation of all pages."""
    import numpy as np

    lens = np.asarray(lengths if lengths is not None else rng.integers(lo, hi + 1, size=requests), dtype=np.int64)
    npages = (lens + page_size - 1) // page_size
    maxp = int(max_pages if max_pages is not None else max(1, int(npages.max(initial=1))))
    total = int(npages.sum())
    perm = rng.permutation(max(total, 1)).astype(np.int32)
    pt = np.zeros((requests, maxp), dtype=np.int32)
    off = 0
    for r in range(requests):
        pt[r, : npages[r]] = perm[off: off + npages[r]]
        off += int(npages[r])
    q = rng.standard_normal((requests, kv_heads, group, head_dim), dtype=np.float32).astype(np.float16)
    kc = rng.standard_normal((max(total, 1), page_size, kv_heads, head_dim), dtype=np.float32).astype(np.float16)
    vc = rng.standard_normal((max(total, 1), page_size, kv_heads, head_dim), dtype=np.float32).astype(np.float16)
    kl = lens.astype(np.int32).reshape(requests, 1)
    out = np.zeros((requests, kv_heads, group, head_dim), dtype=np.float16)
    plan = decode_plan(requests, kv_heads, group, head_dim, max(total, 1), maxp, page_size)
    return plan, [q, kc, vc, pt, kl, out]


def indexer_inputs(rng, batch: int, context: int, topk: int, queries: int = 8, heads: int = 64, head_dim: int = 128):
    """q, k ~ N(0,1) f16; w ~ U(0,1) f32."""
    import numpy as np

    q = rng.standard_normal((batch, queries * heads, head_dim), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((batch, context, head_dim), dtype=np.float32).astype(np.float16)
    w = rng.uniform(0, 1, (batch, queries, heads)).astype(np.float32)
    s = np.zeros((batch, queries, context), np.float32)
    idx = np.zeros((batch, queries, topk), np.int32)
    return indexer_plan(batch, queries, heads, head_dim, context, topk), [q, k, w, s, idx]
