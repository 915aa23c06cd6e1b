"""ctypes wrapper of oracle/cpu_kernels.c (TEST / BASELINE INFRASTRUCTURE ONLY)."""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libptowsp_oracle.so"
_lib = None


def load() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            subprocess.run(["make", "-C", str(HERE), "oracle"], check=True, capture_output=True)
        _lib = C.CDLL(str(LIB))
        _lib.oracle_row_tiles.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int]
        _lib.oracle_gemm_tiles.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int,
                                           C.c_int64, C.c_int64, C.c_int64, C.c_int]
        _lib.oracle_paged_decode.argtypes = [C.c_void_p] * 6 + [C.c_int] * 7
        _lib.oracle_indexer.argtypes = [C.c_void_p] * 5 + [C.c_int] * 7
    return _lib


def threads() -> int:
    return len(os.sched_getaffinity(0))


def row_tiles(kind: str, x: np.ndarray, y: np.ndarray, rows: int, cols: int, nthreads: int | None = None) -> None:
    """kind 'rmsnorm' | 'softmax' over contiguous f32 tiles [..., rows, cols]."""
    assert x.dtype == np.float32 and x.flags.c_contiguous and y.flags.c_contiguous
    nt = x.size // (rows * cols)
    load().oracle_row_tiles(0 if kind == "rmsnorm" else 1, x.ctypes.data, y.ctypes.data, nt, rows, cols,
                            nthreads or threads())


def gemm_tiles(a: np.ndarray, b: np.ndarray, c: np.ndarray, tile_m: int, tile_n: int,
               nthreads: int | None = None) -> None:
    """C[b] = A[b] @ B[b] by 128x128-style output tiles: a [B,M,K] f16, b [B,K,N] f16, c [B,M,N] f32."""
    Bn, M, K = a.shape
    N = b.shape[2]
    base = np.concatenate([a.reshape(-1).view(np.uint16), b.reshape(-1).view(np.uint16)])
    boff = a.size
    offs = []
    for bi in range(Bn):
        for i in range(M // tile_m):
            for j in range(N // tile_n):
                offs += [bi * M * K + i * tile_m * K, boff + bi * K * N + j * tile_n, bi * M * N + i * tile_m * N + j * tile_n]
    offs = np.asarray(offs, dtype=np.int64)
    load().oracle_gemm_tiles(base.ctypes.data, offs.ctypes.data, c.ctypes.data, len(offs) // 3, tile_m, tile_n, K,
                             K, N, N, nthreads or threads())


def paged_decode(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, pt: np.ndarray, lens: np.ndarray, out: np.ndarray,
                 page_size: int, nthreads: int | None = None) -> None:
    """Paged GQA decode over contiguous q/out [R,KVH,G,D] f16, caches [pages,PS,KVH,D] f16, page table [R,maxp]."""
    R, KVH, G, D = q.shape
    arrs = [np.ascontiguousarray(a) for a in (q, kc, vc)]
    pt = np.ascontiguousarray(pt, dtype=np.int32)
    lens = np.ascontiguousarray(np.asarray(lens).reshape(-1), dtype=np.int32)
    assert out.flags.c_contiguous and out.dtype == np.float16 and G <= 8 and D <= 256
    load().oracle_paged_decode(arrs[0].ctypes.data, arrs[1].ctypes.data, arrs[2].ctypes.data, pt.ctypes.data,
                               lens.ctypes.data, out.ctypes.data, R, KVH, G, D, page_size, pt.shape[1],
                               nthreads or threads())


def indexer(q: np.ndarray, k: np.ndarray, w: np.ndarray, s: np.ndarray, idx: np.ndarray, heads: int,
            nthreads: int | None = None) -> None:
    """Scores s [B,Q,T] f32 and stable top-K indices idx [B,Q,K] i32 of q [B,Q*H,D] f16, k [B,T,D], w [B,Q,H]."""
    B, QH, D = q.shape
    T = k.shape[1]
    Q, K = s.shape[1], idx.shape[2]
    q, k, w = (np.ascontiguousarray(a) for a in (q, k, w))
    assert s.flags.c_contiguous and idx.flags.c_contiguous and QH == Q * heads
    load().oracle_indexer(q.ctypes.data, k.ctypes.data, w.ctypes.data, s.ctypes.data, idx.ctypes.data, B, Q, heads, D,
                          T, K, nthreads or threads())
