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
