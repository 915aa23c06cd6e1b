"""The five BASELINE workloads written with the reference's own Python API.

Used (build container only) to check that ``pto_wsp_b200.workloads`` builds the
same plans as ``workload_to_codegen_ir`` + ``module_to_plan``.
"""


import numpy as np


def rmsnorm(B, T, R=16, Cc=128):
    from pto_wsp import DType, Dense, DispatchPolicy, In, Out, P, TaskWindow, Tensor, Tile, WindowMode, kernel, pto, workload
    f32 = DType.F32
    X = Tensor(data=None, shape=(B, T, R, Cc), dtype=f32)
    Y = Tensor(data=None, shape=(B, T, R, Cc), dtype=f32)

    @kernel
    def rmsnorm_tile(x: In[Tile[R, Cc, f32]], out: Out[Tile[R, Cc, f32]]):
        sq = pto.mul(x, x)
        mean_sq = pto.rowmean(sq)
        inv = pto.rsqrt(mean_sq)
        pto.store(out, pto.mul(x, inv))

    @workload
    def rmsnorm():
        for b in P(Dense[B]()):
            for t in P(Dense[T]()):
                rmsnorm_tile[b, t](x=X[b][t], out=Y[b][t])

    return rmsnorm().dispatch(DispatchPolicy.round_robin(num_aicpus=4)).task_graph(
        window=TaskWindow(8192, "tasks", WindowMode.STALL)), [X, Y]


def softmax(B, T, R=32, Cc=256):
    from pto_wsp import DType, Dense, DispatchPolicy, In, Out, P, TaskWindow, Tensor, Tile, WindowMode, kernel, pto, workload
    f32 = DType.F32
    X = Tensor(data=None, shape=(B, T, R, Cc), dtype=f32)
    Y = Tensor(data=None, shape=(B, T, R, Cc), dtype=f32)

    @kernel
    def softmax_tile(x: In[Tile[R, Cc, f32]], out: Out[Tile[R, Cc, f32]]):
        m = pto.rowmax(x)
        e = pto.exp(pto.sub(x, m))
        s = pto.rowsum(e)
        pto.store(out, pto.div(e, s))

    @workload
    def softmax():
        for b in P(Dense[B]()):
            for t in P(Dense[T]()):
                softmax_tile[b, t](x=X[b][t], out=Y[b][t])

    return softmax().dispatch(DispatchPolicy.round_robin(num_aicpus=4)).task_graph(
        window=TaskWindow(8192, "tasks", WindowMode.STALL)), [X, Y]


def bgemm(B, M, N, K, tm=128, tn=128, accumulate=False):
    from pto_wsp import DType, Dense, DispatchPolicy, In, InOut, Out, P, TaskWindow, Tensor, Tile, WindowMode, kernel, pto, workload
    f16, f32 = DType.F16, DType.F32
    A = Tensor(data=None, shape=(B, M // tm, tm, K), dtype=f16)
    Bt = Tensor(data=None, shape=(B, N // tn, K, tn), dtype=f16)
    Cc = Tensor(data=None, shape=(B, M // tm, N // tn, tm, tn), dtype=f32)
    if accumulate:
        @kernel
        def gemm_tile(a: In[Tile[tm, K, f16]], b: In[Tile[K, tn, f16]], c: InOut[Tile[tm, tn, f32]]):
            pto.store(c, pto.add(c, pto.matmul(a, b)))
    else:
        @kernel
        def gemm_tile(a: In[Tile[tm, K, f16]], b: In[Tile[K, tn, f16]], c: Out[Tile[tm, tn, f32]]):
            pto.store(c, pto.matmul(a, b))

    @workload
    def bgemm():
        for b in P(Dense[B]()):
            for i in P(Dense[M // tm]()):
                for j in P(Dense[N // tn]()):
                    gemm_tile[b, i, j](a=A[b][i], b=Bt[b][j], c=Cc[b][i][j])

    return bgemm().dispatch(DispatchPolicy.round_robin(num_aicpus=4)).task_graph(
        window=TaskWindow(8192, "tasks", WindowMode.STALL)), [A, Bt, Cc]


def decode(R, KVH, G, D, pages, maxp, page_size=16):
    from pto_wsp import DType, Dense, DenseDyn, DispatchPolicy, In, Out, P, Scalar, TaskWindow, Tensor, Tile, WindowMode, kernel, workload
    from pto_wsp_b200.workloads import PAGED_DECODE_CPU_BODY
    f16, i32 = DType.F16, DType.I32
    Q = Tensor(data=None, shape=(R, KVH, G, D), dtype=f16)
    KC = Tensor(data=None, shape=(pages, page_size, KVH, D), dtype=f16)
    VC = Tensor(data=None, shape=(pages, page_size, KVH, D), dtype=f16)
    PT = Tensor(data=None, shape=(R, maxp), dtype=i32)
    KL = Tensor(data=None, shape=(R, 1), dtype=i32)
    O = Tensor(data=None, shape=(R, KVH, G, D), dtype=f16)

    @kernel(cpp_src=PAGED_DECODE_CPU_BODY)
    def paged_decode(q: In[Tile[G, D, f16]], k_cache: In[Tile[page_size, KVH * D, f16]],
                     v_cache: In[Tile[page_size, KVH * D, f16]], page_table: In[Tile[1, maxp, i32]],
                     kv_len: In[Tile[1, 1, i32]], out: Out[Tile[G, D, f16]],
                     page_size: Scalar[i32] = page_size, num_kv_heads: Scalar[i32] = KVH):
        pass

    @workload
    def paged():
        for b in P(DenseDyn(R)):
            for h in P(Dense[KVH]()):
                paged_decode[b, h](q=Q[b][h], k_cache=KC, v_cache=VC, page_table=PT[b], kv_len=KL[b], out=O[b][h])

    return paged().dispatch(DispatchPolicy.round_robin(num_aicpus=4)).task_graph(
        window=TaskWindow(8192, "tasks", WindowMode.STALL)), [Q, KC, VC, PT, KL, O]


def indexer(B, Qn, H, D, T, K):
    from pto_wsp import DType, Dense, DispatchPolicy, In, Out, P, TaskWindow, Tensor, Tile, WindowMode, kernel, workload
    from pto_wsp_b200.workloads import INDEXER_SCORE_CPU_BODY, TOPK_CPU_BODY
    f16, f32, i32 = DType.F16, DType.F32, DType.I32
    Qt = Tensor(data=None, shape=(B, Qn * H, D), dtype=f16)
    Kt = Tensor(data=None, shape=(B, T, D), dtype=f16)
    W = Tensor(data=None, shape=(B, Qn, H), dtype=f32)
    S = Tensor(data=None, shape=(B, Qn, T), dtype=f32)
    I = Tensor(data=None, shape=(B, Qn, K), dtype=i32)

    @kernel(cpp_src=INDEXER_SCORE_CPU_BODY)
    def indexer_score(q: In[Tile[Qn * H, D, f16]], k: In[Tile[T, D, f16]], w: In[Tile[Qn, H, f32]],
                      scores: Out[Tile[Qn, T, f32]]):
        pass

    @kernel(cpp_src=TOPK_CPU_BODY)
    def topk(scores: In[Tile[1, T, f32]], out: Out[Tile[1, K, i32]]):
        pass

    @workload
    def lightning_indexer():
        for b in P(Dense[B]()):
            indexer_score[b](q=Qt[b], k=Kt[b], w=W[b], scores=S[b])
        for b2 in P(Dense[B]()):
            for q in P(Dense[Qn]()):
                topk[b2, q](scores=S[b2][q], out=I[b2][q])

    return lightning_indexer().dispatch(DispatchPolicy.round_robin(num_aicpus=4)).task_graph(
        window=TaskWindow(8192, "tasks", WindowMode.STALL)), [Qt, Kt, W, S, I]
