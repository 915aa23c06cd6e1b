"""Runs the reference's own CPU-sim artifacts of the five configs on the host cores (TEST / BASELINE
INFRASTRUCTURE ONLY: ``bench.py --impl reference``).

The artifacts (oracle/build_artifacts.py) are the reference's generated ``<module>_main`` task loops and kernels,
loaded and called through the reference's own ``CodegenExecutable`` from its IR module in oracle/_ref
(``run_with_symbols``, ``src/python/pto_codegen.cpp:3510-3576``) -- the stock CPU-sim path.  That path is
single-threaded by construction (the task loop runs on the calling thread), so, as the CPU-sim's own answer to
using every core, the host runs one process per core, each with its share of the config's outer-axis units
(independent by the loop nest, so the split changes no result).  A step sends every worker one "go" and waits for
all of them; its time is the slowest worker's.
"""

from __future__ import annotations

import json
import os
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
ART = HERE / "_ref" / "artifacts"

_DT = {"f32": "float32", "f16": "float16", "i32": "int32", "i64": "int64"}


def manifest() -> dict | None:
    p = ART / "manifest.json"
    if not p.exists() or not list((HERE / "_ref").glob("pto_ir_cpp*.so")):
        return None
    m = json.loads(p.read_text())
    return m if all((ART / v["so"]).exists() for v in m.values()) else None


def unit_inputs(name: str, unit: dict, seed: int):
    """Seeded inputs of one unit (BASELINE.json distributions), as the artifact's tensors, plus its axis sizes."""
    import numpy as np

    rng = np.random.default_rng(seed)
    tensors = manifest()[name]["tensors"]
    if name == "decode":
        L = int(unit["length"])
        npages = max(1, (L + 15) // 16)
        q = rng.standard_normal((1, 8, 4, 128), dtype=np.float32).astype(np.float16)
        kc = rng.standard_normal((npages, 16, 8, 128), dtype=np.float32).astype(np.float16)
        vc = rng.standard_normal((npages, 16, 8, 128), dtype=np.float32).astype(np.float16)
        pt = np.zeros(tensors[3]["shape"], np.int32)
        pt[0, :npages] = np.arange(npages, dtype=np.int32)
        kl = np.full((1, 1), L, np.int32)
        out = np.zeros((1, 8, 4, 128), np.float16)
        return [q, kc, vc, pt, kl, out], {"b": 1}
    arrays = []
    for i, t in enumerate(tensors):
        shape, dt = tuple(t["shape"]), np.dtype(_DT[t["dtype"]])
        if name == "softmax" and i == 0:
            a = rng.standard_normal(shape, dtype=np.float32) * 4.0
            a[rng.random(shape, dtype=np.float32) < 0.01] = 30.0
        elif name in ("softmax", "rmsnorm") and i == 0 or name == "indexer" and i in (0, 1):
            a = rng.standard_normal(shape, dtype=np.float32)
        elif name == "bgemm" and i in (0, 1):
            a = rng.uniform(-1, 1, shape)
        elif name == "indexer" and i == 2:
            a = rng.uniform(0, 1, shape)
        else:
            a = np.zeros(shape)
        arrays.append(np.ascontiguousarray(a.astype(dt)))
    return arrays, {}


def _worker(conn, name: str, units: list[dict], seed: int) -> None:
    sys.path.insert(0, str(HERE / "_ref"))
    import pto_ir_cpp

    m = manifest()[name]
    ex = pto_ir_cpp.CodegenExecutable(str(ART / m["so"]), m["entrypoint"])
    inputs = [unit_inputs(name, u, seed + int(u["index"])) for u in units]
    conn.send(("ready", 0.0, 0))
    while True:
        msg = conn.recv()
        if msg != "go":
            break
        t0 = time.perf_counter()
        cycles = 0
        for arrays, axis in inputs:
            cycles += int(ex.run_with_symbols(arrays, axis, {}, {}))
        conn.send(("done", time.perf_counter() - t0, cycles))
    conn.close()


class Pool:
    """`procs` worker processes (spawned: no CUDA or thread state is inherited) sharing `units` round-robin."""

    def __init__(self, name: str, units: list[dict], procs: int, seed: int = 0):
        import multiprocessing as mp

        ctx = mp.get_context("spawn")
        self.procs = max(1, min(procs, len(units)))
        self.conns, self.ps = [], []
        for w in range(self.procs):
            a, b = ctx.Pipe()
            p = ctx.Process(target=_worker, args=(b, name, units[w::self.procs], seed), daemon=True)
            p.start()
            self.conns.append(a)
            self.ps.append(p)
        for c in self.conns:
            c.recv()  # ready: inputs generated, artifact loaded

    def step(self) -> tuple[float, list[float]]:
        t0 = time.perf_counter()
        for c in self.conns:
            c.send("go")
        times = [c.recv()[1] for c in self.conns]
        return time.perf_counter() - t0, times

    def close(self) -> None:
        for c in self.conns:
            try:
                c.send("stop")
            except (BrokenPipeError, OSError):
                pass
        for p in self.ps:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()


def host_cores() -> int:
    return len(os.sched_getaffinity(0))
