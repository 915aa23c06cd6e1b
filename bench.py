#!/usr/bin/env python3
"""Benchmark of the PTO-WSP cuda_sm100a task loop: all five BASELINE configs, one JSON line on rank 0.

A *step* is one pass of the task loop over one whole config (its global batch).  The headline line is config 2
(row softmax, X[32,2048,32,256] f32); configs 1, 3, 4 and 5 ride in the same line under ``workloads``, each with
its own ``value``, ``ms_per_step``, ``roofline``, ``e2e``, ``cpu_baseline`` and ``clocks``.  ``--workload NAME``
runs one config alone.

* ``value`` -- whole-job throughput (algorithmic GB/s or TFLOP/s, formulas per config below) with every input
  already in HBM: K back-to-back steps through ``ShardedExecutable.run_with_symbols`` (the reference-facing
  ``CodegenExecutable`` surface over the C ABI), timed with CUDA events on the launch stream between a barrier +
  synchronize on both sides, max over ranks.  Every config's inputs exceed L2 (126 MB) except config 5's keys
  (128 MiB), so no flush is needed.
* ``e2e``   -- the same metric through the same call with pinned host numpy buffers: each step stages the
  inputs host->device and the outputs device->host (bytes per step from the runtime's own counters).
* ``roofline`` -- the dominant kernel: its algorithmic work per launch / its average launch time, measured with
  CUDA events bracketing each of its launches on the launch stream (runtime option ``kernel_events``) over a
  second pass of the same K steps, right after the first, inside the clock-sampled region (the event records would
  stretch the steps of the ``value`` pass), against the measured peak in MEASURED_PEAKS.json; ``traffic`` = ncu
  DRAM bytes per launch from profiles/traffic.json (scaled to this rank's share of the units).
* ``cpu_baseline`` -- the C port of the CPU-sim task bodies (oracle/cpu_kernels.c) on the host cores, rank 0 at
  N=1, bounded sample.
* ``--impl reference`` -- the reference arm: the reference's own CPU-sim artifact of each config (its generated
  task loop and kernels, oracle/_ref, built with the clean-room pto-isa stand-in) through its own
  ``CodegenExecutable``, one single-threaded process per host core, same metric and config, one line with the same
  ``workloads`` layout; rank 0 only.  Without the built artifacts it times the C port instead.

Multi-GPU (torchrun, one rank per GPU): every rank runs its ``ShardedExecutable`` share of the ONE global config
(strong scaling): contiguous blocks of the outer ``P(batch)`` axis for configs 1, 2, 3 and 5, contiguous blocks
balanced by KV length for config 4 (``--partition`` overrides).  No data-path collective: NCCL carries only the
barriers and the max-over-ranks timing.

Algorithmic work per step (global):
  1 RMSNorm   8 B per element (read x, write y), 64 x 4096 x 16 x 128 elements
  2 softmax   8 B per element, 32 x 2048 x 32 x 256 elements
  3 bgemm     2 M N K flop per batch element, 64 x 2048^3
  4 decode    K + V bytes of every request's tokens (L x 8 heads x 128 x 2 B x 2) + Q and O (64 x 32 x 128 x 2 B x 2)
  5 indexer   scoring flop 2 x 512 x 128 per key per batch element (16 x 32768 keys); the top-k runs in the step
"""

from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ORDER = ["softmax", "rmsnorm", "bgemm", "decode", "indexer"]  # the first is the headline


def _env_int(k: str, d: int) -> int:
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def peaks(key: str = "hbm_gbs") -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())[key]), "measured"
        except Exception:  # noqa: BLE001
            pass
    return (6650.0 if key == "hbm_gbs" else 1590.0), "fallback"


def traffic_from_profiles(key: str) -> float | None:
    """ncu DRAM bytes of one full-config launch of the dominant kernel (profiles/traffic.json)."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        v = json.loads(p.read_text()).get(key)
        return float(v["bytes_per_launch"]) if v else None
    except Exception:  # noqa: BLE001
        return None


# ---------------------------------------------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------------------------------------------


class NvmlClockSampler:
    """SM clock, power and clock-event reasons read through NVML every millisecond while the timed region runs
    (read-only queries).  Falls back to nvidia-smi."""

    REASONS = [("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap")]

    def __init__(self, gpu_index: int, pci_bus_id: str | None = None):
        self.idx, self.pci = gpu_index, pci_bus_id
        self.fallback = None
        self.rows: list[tuple[float, float, float, int]] = []

    def __enter__(self):
        try:
            import pynvml as N

            N.nvmlInit()
            self.N = N
            h = None
            if self.pci:
                try:
                    h = N.nvmlDeviceGetHandleByPciBusId(self.pci)
                except Exception:  # noqa: BLE001
                    h = None
            self.h = h if h is not None else N.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = float(N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM))
            self.stop = threading.Event()
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception:  # noqa: BLE001
            self.fallback = ClockSampler(self.idx).__enter__()
        return self

    def _run(self):
        N = self.N
        while not self.stop.is_set():
            try:
                self.rows.append((float(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM)), self.max_mhz,
                                  N.nvmlDeviceGetPowerUsage(self.h) / 1000.0,
                                  int(N.nvmlDeviceGetCurrentClocksEventReasons(self.h))))
            except Exception:  # noqa: BLE001
                break
            time.sleep(0.001)

    def __exit__(self, *a):
        if self.fallback is not None:
            self.fallback.__exit__(*a)
            return
        self.stop.set()
        self.thread.join(timeout=5)

    def summary(self) -> dict:
        if self.fallback is not None:
            return self.fallback.summary()
        reasons = set()
        for _, _, _, bits in self.rows:
            for name, attr in self.REASONS:
                if bits & getattr(self.N, attr, 0):
                    reasons.add(name)
        sm = [r[0] for r in self.rows]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples_under_load": len(sm), "samples": len(sm), "source": "nvml, 1 ms",
                "power_w_max": round(max((r[2] for r in self.rows), default=0.0), 1)}


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:  # noqa: BLE001
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()

    def summary(self) -> dict:
        rows = [r for r in csv.reader(io.StringIO(getattr(self, "out", ""))) if len(r) >= 9]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                s, m, pw = float(r[1]), float(r[2]), float(r[3])
            except ValueError:
                continue
            mx = m
            if pw > 250.0:  # under load
                sm.append(s)
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples_under_load": len(sm), "samples": len(rows)}


def _pci_bus_id(torch, dev) -> str | None:
    try:
        p = torch.cuda.get_device_properties(dev)
        return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
    except Exception:  # noqa: BLE001
        return None


def gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = [p for p in vis.split(",") if p.strip()]
        if local_rank < len(parts) and parts[local_rank].strip().isdigit():
            return int(parts[local_rank])
    return local_rank


def _cpu_native():
    sys.path.insert(0, str(ROOT / "oracle"))
    import cpu_native

    return cpu_native


# ---------------------------------------------------------------------------------------------------------------
# the five configs
# ---------------------------------------------------------------------------------------------------------------


class Case:
    """One BASELINE config: its global plan, seeded inputs, work formula, shard method and CPU legs."""

    name = ""
    unit = "GB/s"
    bound = "hbm"
    dtype = "f32"
    kernel = ""          # plan kernel name of the dominant kernel
    traffic_key = ""     # profiles/traffic.json key (full-config launch)
    method = "block"

    def __init__(self, args):
        self.args = args

    @property
    def scale(self) -> float:
        return 1e9 if self.unit == "GB/s" else 1e12

    def costs(self):
        return None

    def axis(self, n_local: int | None = None) -> dict:
        return {}

    def outputs(self, darr) -> list:
        return []

    def unit_work(self, units: list[int]) -> float:
        """Algorithmic work of the dominant kernel over these outer-axis units (one launch per step)."""
        return self.work() * len(units) / self.n_units

    def check(self, darr) -> dict:
        return {}


class RowCase(Case):
    rows = cols = 0
    batch = tiles = 0

    def __init__(self, args):
        super().__init__(args)
        if args.batch:
            self.batch = args.batch
        if args.cols:
            self.cols = args.cols
        self.n_units = self.batch

    @property
    def config(self) -> str:
        return (f"{self.cfg_name}: X[{self.batch},{self.tiles},{self.rows},{self.cols}] f32, Tile[{self.rows},"
                f"{self.cols}], P(batch) x P(tiles)")

    def elems(self) -> int:
        return self.batch * self.tiles * self.rows * self.cols

    def work(self) -> float:
        return float(self.elems() * 8)

    def plan(self):
        from pto_wsp_b200 import workloads

        fn = workloads.softmax_plan if self.name == "softmax" else workloads.rmsnorm_plan
        return fn(self.batch, self.tiles, self.rows, self.cols)

    def device_inputs(self, torch, dev):
        g = torch.Generator(device=dev)
        g.manual_seed(self.seed)
        shape = (self.batch, self.tiles, self.rows, self.cols)
        x = torch.randn(shape, generator=g, device=dev, dtype=torch.float32)
        if self.name == "softmax":
            x *= 4.0
            x[torch.rand(shape, generator=g, device=dev) < 0.01] = 30.0
        return [x, torch.empty_like(x)]

    def outputs(self, darr):
        return [1]

    def check(self, darr) -> dict:
        import numpy as np

        x, y = darr
        xs = x.reshape(-1, self.rows, self.cols)[:64].double().cpu().numpy()
        ys = y.reshape(-1, self.rows, self.cols)[:64].double().cpu().numpy()
        if self.name == "softmax":
            ref = np.exp(xs - xs.max(-1, keepdims=True))
            ref /= ref.sum(-1, keepdims=True)
        else:
            ref = xs / np.sqrt((xs * xs).mean(-1, keepdims=True))
        return {"max_rel_err_vs_fp64_64_tiles": float(np.max(np.abs(ys - ref) / (np.abs(ref) + 1e-30)))}

    def _tiles(self, hx, n: int):
        import numpy as np

        return np.ascontiguousarray(hx.reshape(-1, self.rows, self.cols)[:n])

    def cpu_baseline(self, host, budget_s: float) -> dict:
        import numpy as np

        cn = _cpu_native()
        nth = cn.threads()
        total = self.batch * self.tiles
        n = min(total, 4096)
        x = self._tiles(host[0], n)
        y = np.empty_like(x)
        t0 = time.perf_counter()
        cn.row_tiles(self.name, x, y, self.rows, self.cols, nth)
        dt = time.perf_counter() - t0
        n2 = int(min(total, max(n, n * budget_s / max(dt, 1e-6) * 0.5)))
        x = self._tiles(host[0], n2)
        y = np.empty_like(x)
        t0 = time.perf_counter()
        cn.row_tiles(self.name, x, y, self.rows, self.cols, nth)
        dt = time.perf_counter() - t0
        return {"value": round(n2 * self.rows * self.cols * 8 / dt / 1e9, 3), "unit": "GB/s", "cores": nth,
                "kind": "port", "sample": f"{n2} of {total} tiles ({n2 * self.rows * self.cols * 4 / 2**20:.0f} MiB "
                                          f"in), {dt:.2f} s, C port of the CPU-sim tile loop (oracle/cpu_kernels.c)"}

    def reference(self, steps: int, warmup: int) -> dict:
        """The whole config per step (all tiles), C port on all host threads."""
        import numpy as np

        cn = _cpu_native()
        nth = cn.threads()
        total = self.batch * self.tiles
        rng = np.random.default_rng(self.seed)
        x = np.empty((total, self.rows, self.cols), np.float32)
        for t0 in range(0, total, 4096):  # in slices: the mask of the whole tensor would take 4 GiB
            xs = x[t0:t0 + 4096]
            xs[...] = rng.standard_normal(xs.shape, dtype=np.float32)
            if self.name == "softmax":
                xs *= 4.0
                xs[rng.random(xs.shape, dtype=np.float32) < 0.01] = 30.0
        y = np.empty_like(x)
        for _ in range(warmup):
            cn.row_tiles(self.name, x, y, self.rows, self.cols, nth)
        t0 = time.perf_counter()
        for _ in range(steps):
            cn.row_tiles(self.name, x, y, self.rows, self.cols, nth)
        dt = time.perf_counter() - t0
        v = self.work() * steps / dt / 1e9
        return {"value": round(v, 3), "unit": "GB/s", "steps": steps, "ms_per_step": round(dt / steps * 1e3, 3),
                "same_config": True, "cpu_baseline": {
                    "value": round(v, 3), "unit": "GB/s", "cores": nth, "kind": "port",
                    "sample": f"the whole config per step ({total} tiles); C port of the CPU-sim tile loop "
                              f"(oracle/cpu_kernels.c), {nth} threads"}}


class SoftmaxCase(RowCase):
    name, cfg_name, kernel, traffic_key = "softmax", "config 2: row softmax", "softmax_tile", "softmax:softmax_rows"
    batch, tiles, rows, cols, seed = 32, 2048, 32, 256, 1000
    metric = "row-softmax task-loop throughput (algorithmic HBM bytes)"


class RmsNormCase(RowCase):
    name, cfg_name, kernel, traffic_key = "rmsnorm", "config 1: RMSNorm (GPU scale)", "rmsnorm_tile", "rmsnorm:rmsnorm_rows"
    batch, tiles, rows, cols, seed = 64, 4096, 16, 128, 1001
    metric = "RMSNorm task-loop throughput (algorithmic HBM bytes)"


class BgemmCase(Case):
    name, kernel, traffic_key = "bgemm", "gemm_tile", "bgemm:matmul_tcgen05"
    unit, bound, dtype = "TFLOP/s", "tensor", "f16 in / f32 acc"
    metric = "bgemm task-loop throughput"
    B, M, N, K = 64, 2048, 2048, 2048

    def __init__(self, args):
        super().__init__(args)
        if args.batch:
            self.B = args.batch
        self.n_units = self.B

    @property
    def config(self) -> str:
        return (f"config 3: bgemm {self.B} x ({self.M}x{self.N}x{self.K}), f16 in, f32 acc/out, 128x128 output tiles, "
                f"K inside the kernel")

    def work(self) -> float:
        return 2.0 * self.B * self.M * self.N * self.K

    def plan(self):
        from pto_wsp_b200 import workloads

        return workloads.bgemm_plan(self.B, self.M, self.N, self.K)

    def device_inputs(self, torch, dev):
        from pto_wsp_b200 import workloads

        g = torch.Generator(device=dev)
        g.manual_seed(2000)
        self._abc = ((torch.rand((self.B, self.M, self.K), generator=g, device=dev) * 2 - 1).half(),
                     (torch.rand((self.B, self.K, self.N), generator=g, device=dev) * 2 - 1).half(),
                     torch.empty((self.B, self.M, self.N), device=dev, dtype=torch.float32))
        return list(workloads.bgemm_views(*self._abc))

    def host_views(self, torch):
        """Pinned host copies of A, B, C and the plan's views of them."""
        from pto_wsp_b200 import workloads

        hs = []
        for t in self._abc:
            h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            h.copy_(t)
            hs.append(h.numpy())
        self._host_abc = hs
        return list(workloads.bgemm_views(*hs))

    def outputs(self, darr):
        return [2]

    def check(self, darr) -> dict:
        a, b, c = self._abc
        ref = a[0].double() @ b[0].double()
        big = ref.abs() > 1e-2 * ref.abs().max()
        rel = ((c[0].double() - ref).abs() / ref.abs())[big]
        return {"max_rel_err_vs_fp64_batch0": float(rel.max())}

    def cpu_baseline(self, host, budget_s: float) -> dict:
        import numpy as np

        cn = _cpu_native()
        nth = cn.threads()
        a, b = self._host_abc[0], self._host_abc[1]
        rows = 128
        c = np.empty((1, rows, self.N), np.float32)
        t0 = time.perf_counter()
        cn.gemm_tiles(a[:1, :rows], b[:1], c, 128, 128, nth)
        dt = time.perf_counter() - t0
        reps = max(1, min(int(budget_s / max(dt, 1e-6)), self.M // rows))
        rows2 = rows * reps
        c = np.empty((1, rows2, self.N), np.float32)
        t0 = time.perf_counter()
        cn.gemm_tiles(np.ascontiguousarray(a[:1, :rows2]), b[:1], c, 128, 128, nth)
        dt = time.perf_counter() - t0
        return {"value": round(2.0 * rows2 * self.N * self.K / dt / 1e12, 6), "unit": "TFLOP/s", "cores": nth,
                "kind": "port", "sample": f"{rows2}x{self.N}x{self.K} rows of batch element 0 ({dt:.2f} s), C port "
                                          f"of the CPU-sim gemm tile task (oracle/cpu_kernels.c, f32 accumulation)"}

    def reference(self, steps: int, warmup: int) -> dict:
        import numpy as np

        cn = _cpu_native()
        nth = cn.threads()
        rng = np.random.default_rng(0)
        rows = 512
        a = rng.uniform(-1, 1, (1, rows, self.K)).astype(np.float16)
        b = rng.uniform(-1, 1, (1, self.K, self.N)).astype(np.float16)
        c = np.empty((1, rows, self.N), np.float32)
        for _ in range(min(warmup, 1)):
            cn.gemm_tiles(a, b, c, 128, 128, nth)
        t0 = time.perf_counter()
        for _ in range(steps):
            cn.gemm_tiles(a, b, c, 128, 128, nth)
        dt = time.perf_counter() - t0
        v = 2.0 * rows * self.N * self.K * steps / dt / 1e12
        return {"value": round(v, 6), "unit": "TFLOP/s", "steps": steps, "ms_per_step": round(dt / steps * 1e3, 3),
                "same_config": False, "cpu_baseline": {
                    "value": round(v, 6), "unit": "TFLOP/s", "cores": nth, "kind": "port",
                    "sample": f"a {rows}x{self.N}x{self.K} slab (4 of 16 m-tile rows of one batch element) per step; "
                              f"the full config is {self.B * self.M // rows}x that; C port of the CPU-sim gemm tile "
                              f"task, {nth} threads"}}


class DecodeCase(Case):
    # contiguous shares balanced by KV length: the rank works on views of the global tensors.  (LPT balances a
    # little better, but its non-contiguous shares cost a gather of Q / page table / lengths and a scatter of the
    # output per step: 0.141 against 0.112 ms per step at 2 ranks.)
    name, kernel, traffic_key, method = "decode", "paged_decode", "decode:paged_decode_tma", "balanced"
    unit, bound, dtype = "GB/s", "hbm", "f16 in / f32 softmax / f16 out"
    metric = "paged GQA decode task-loop throughput (algorithmic HBM bytes)"
    R, KVH, G, D, PS = 64, 8, 4, 128, 16

    def __init__(self, args):
        super().__init__(args)
        import numpy as np

        if args.batch:
            self.R = args.batch
        self.n_units = self.R
        rng = np.random.default_rng(3000)
        self.lens = rng.integers(512, 8192 + 1, size=self.R).astype(np.int64)
        self.npages = (self.lens + self.PS - 1) // self.PS
        self.maxp = int(self.npages.max())
        self.total_pages = int(self.npages.sum())
        perm = rng.permutation(self.total_pages).astype(np.int32)
        self.pt = np.zeros((self.R, self.maxp), np.int32)
        off = 0
        for r in range(self.R):
            self.pt[r, : self.npages[r]] = perm[off: off + self.npages[r]]
            off += int(self.npages[r])

    @property
    def config(self) -> str:
        return (f"config 4: paged GQA decode, {self.R} requests, 32 q / 8 kv heads, d=128, f16, page 16, KV len "
                f"U[512,8192] (sum {int(self.lens.sum())} tokens), random page permutation")

    def costs(self):
        return [float(x) for x in self.lens]

    def axis(self, n_local=None):
        return {"b": int(n_local if n_local is not None else self.R)}

    def _work(self, units) -> float:
        L = float(self.lens[list(units)].sum())
        return L * self.KVH * self.D * 2 * 2 + len(units) * self.KVH * self.G * self.D * 2 * 2

    def work(self) -> float:
        return self._work(range(self.R))

    def unit_work(self, units):
        return self._work(units)

    def plan(self):
        from pto_wsp_b200 import workloads

        return workloads.decode_plan(self.R, self.KVH, self.G, self.D, self.total_pages, self.maxp, self.PS)

    def device_inputs(self, torch, dev):
        g = torch.Generator(device=dev)
        g.manual_seed(3001)
        q = torch.randn((self.R, self.KVH, self.G, self.D), generator=g, device=dev).half()
        kc = torch.randn((self.total_pages, self.PS, self.KVH, self.D), generator=g, device=dev).half()
        vc = torch.randn((self.total_pages, self.PS, self.KVH, self.D), generator=g, device=dev).half()
        pt = torch.from_numpy(self.pt).to(dev)
        kl = torch.tensor(self.lens.reshape(self.R, 1), dtype=torch.int32, device=dev)
        out = torch.zeros((self.R, self.KVH, self.G, self.D), dtype=torch.float16, device=dev)
        return [q, kc, vc, pt, kl, out]

    def outputs(self, darr):
        return [5]

    def check(self, darr) -> dict:
        import math

        torch = sys.modules["torch"]
        q, kc, vc, pt, kl, out = darr
        worst = 0.0
        for r in (0, self.R // 2, self.R - 1):
            L = int(self.lens[r])
            pages = pt[r, : (L + self.PS - 1) // self.PS].long()
            k = kc[pages].reshape(-1, self.KVH, self.D)[:L].double()
            v = vc[pages].reshape(-1, self.KVH, self.D)[:L].double()
            s = torch.einsum("hgd,thd->hgt", q[r].double(), k) / math.sqrt(self.D)
            ref = torch.einsum("hgt,thd->hgd", torch.softmax(s, -1), v)
            err = ((out[r].double() - ref).abs() / (ref.abs() + ref.pow(2).mean().sqrt())).max()
            worst = max(worst, float(err))
        return {"max_err_vs_fp64_3_requests": worst}

    def _body_sample(self, host, reqs: list[int]):
        """Inputs of a few requests as their own small decode problem (pages renumbered)."""
        import numpy as np

        q, kc, vc, pt, kl, _ = host
        pages = np.concatenate([pt[r, : self.npages[r]] for r in reqs])
        maxp = int(max(self.npages[r] for r in reqs))
        spt = np.zeros((len(reqs), maxp), np.int32)
        off = 0
        for i, r in enumerate(reqs):
            n = int(self.npages[r])
            spt[i, :n] = np.arange(off, off + n, dtype=np.int32)
            off += n
        return (np.ascontiguousarray(q[reqs]), np.ascontiguousarray(kc[pages]), np.ascontiguousarray(vc[pages]), spt,
                self.lens[reqs].astype(np.int32), np.zeros((len(reqs), self.KVH, self.G, self.D), np.float16))

    def cpu_baseline(self, host, budget_s: float) -> dict:
        cn = _cpu_native()
        nth = cn.threads()
        reqs = [0, 1]
        t0 = time.perf_counter()
        s = self._body_sample(host, reqs)
        cn.paged_decode(*s, self.PS, nth)
        dt = time.perf_counter() - t0
        n = int(max(2, min(self.R, len(reqs) * budget_s / max(dt, 1e-6) * 0.5)))
        reqs = list(range(n))
        s = self._body_sample(host, reqs)
        t0 = time.perf_counter()
        cn.paged_decode(*s, self.PS, nth)
        dt = time.perf_counter() - t0
        return {"value": round(self._work(reqs) / dt / 1e9, 4), "unit": "GB/s", "cores": nth, "kind": "port",
                "sample": f"{n} of {self.R} requests x 8 kv heads ({dt:.2f} s), C port of the paged-decode task body "
                          f"(oracle/cpu_kernels.c: online softmax per query head, f32)"}

    def reference(self, steps: int, warmup: int) -> dict:
        import numpy as np

        cn = _cpu_native()
        nth = cn.threads()
        rng = np.random.default_rng(1)
        host = [rng.standard_normal((self.R, self.KVH, self.G, self.D), dtype=np.float32).astype(np.float16),
                rng.standard_normal((self.total_pages, self.PS, self.KVH, self.D), dtype=np.float32).astype(np.float16),
                rng.standard_normal((self.total_pages, self.PS, self.KVH, self.D), dtype=np.float32).astype(np.float16),
                self.pt, self.lens.astype(np.int32).reshape(-1, 1), None]
        reqs = list(range(min(self.R, 16)))
        s = self._body_sample(host, reqs)
        for _ in range(min(warmup, 1)):
            cn.paged_decode(*s, self.PS, nth)
        t0 = time.perf_counter()
        for _ in range(steps):
            cn.paged_decode(*s, self.PS, nth)
        dt = time.perf_counter() - t0
        v = self._work(reqs) * steps / dt / 1e9
        return {"value": round(v, 4), "unit": "GB/s", "steps": steps, "ms_per_step": round(dt / steps * 1e3, 3),
                "same_config": False, "cpu_baseline": {
                    "value": round(v, 4), "unit": "GB/s", "cores": nth, "kind": "port",
                    "sample": f"{len(reqs)} of {self.R} requests x 8 kv heads per step (same lengths and pages); "
                              f"C port of the paged-decode task body, {nth} threads"}}


class IndexerCase(Case):
    name, kernel, traffic_key = "indexer", "indexer_score", "indexer:indexer_score"
    unit, bound, dtype = "TFLOP/s", "tensor", "f16 in / f32 scores / i32 indices"
    metric = "lightning-indexer task-loop throughput (scoring flop; step = scoring + top-2048)"
    B, Q, H, D, T, TOPK = 16, 8, 64, 128, 32768, 2048

    def __init__(self, args):
        super().__init__(args)
        if args.batch:
            self.B = args.batch
        self.n_units = self.B

    @property
    def config(self) -> str:
        return (f"config 5: lightning indexer {self.B} batches x {self.Q} queries, {self.H} heads, d={self.D}, "
                f"{self.T} keys, top-{self.TOPK}")

    def work(self) -> float:
        return 2.0 * self.B * self.Q * self.H * self.D * self.T

    def plan(self):
        from pto_wsp_b200 import workloads

        return workloads.indexer_plan(self.B, self.Q, self.H, self.D, self.T, self.TOPK)

    def device_inputs(self, torch, dev):
        g = torch.Generator(device=dev)
        g.manual_seed(4000)
        q = torch.randn((self.B, self.Q * self.H, self.D), generator=g, device=dev).half()
        k = torch.randn((self.B, self.T, self.D), generator=g, device=dev).half()
        w = torch.rand((self.B, self.Q, self.H), generator=g, device=dev)
        s = torch.zeros((self.B, self.Q, self.T), device=dev)
        idx = torch.zeros((self.B, self.Q, self.TOPK), dtype=torch.int32, device=dev)
        return [q, k, w, s, idx]

    def outputs(self, darr):
        return [3, 4]

    def check(self, darr) -> dict:
        torch = sys.modules["torch"]
        q, k, w, s, idx = darr
        qd = q[0].double().reshape(self.Q, self.H, self.D)
        ref = (torch.relu(torch.einsum("qhd,td->qht", qd, k[0].double())) * w[0].double()[:, :, None]).sum(1)
        err = float(((s[0].double() - ref).abs() / (ref.abs() + ref.abs().mean())).max())
        # the indices must be the stable top-k of the GPU's own scores (score descending, ties -> lower index)
        sc = s[0]
        order = torch.sort(-sc.double(), dim=-1, stable=True).indices[:, : self.TOPK].int()
        exact = bool(torch.equal(order, idx[0]))
        return {"score_err_vs_fp64_batch0": err, "topk_exact_on_gpu_scores_batch0": exact}

    def cpu_baseline(self, host, budget_s: float) -> dict:
        import numpy as np

        cn = _cpu_native()
        nth = cn.threads()
        q, k, w = host[0], host[1], host[2]
        n = 1
        s = np.zeros((n, self.Q, self.T), np.float32)
        idx = np.zeros((n, self.Q, self.TOPK), np.int32)
        t0 = time.perf_counter()
        cn.indexer(q[:n], k[:n], w[:n], s, idx, self.H, nth)
        dt = time.perf_counter() - t0
        n2 = int(max(1, min(self.B, budget_s / max(dt, 1e-6) * 0.5)))
        if n2 > n:
            s = np.zeros((n2, self.Q, self.T), np.float32)
            idx = np.zeros((n2, self.Q, self.TOPK), np.int32)
            t0 = time.perf_counter()
            cn.indexer(q[:n2], k[:n2], w[:n2], s, idx, self.H, nth)
            dt = time.perf_counter() - t0
        return {"value": round(2.0 * n2 * self.Q * self.H * self.D * self.T / dt / 1e12, 6), "unit": "TFLOP/s",
                "cores": nth, "kind": "port",
                "sample": f"{n2} of {self.B} batch elements, scoring + top-{self.TOPK} ({dt:.2f} s), C port of the "
                          f"indexer task bodies (oracle/cpu_kernels.c)"}

    def reference(self, steps: int, warmup: int) -> dict:
        import numpy as np

        cn = _cpu_native()
        nth = cn.threads()
        rng = np.random.default_rng(1)
        n = 1
        q = rng.standard_normal((n, self.Q * self.H, self.D), dtype=np.float32).astype(np.float16)
        k = rng.standard_normal((n, self.T, self.D), dtype=np.float32).astype(np.float16)
        w = rng.uniform(0, 1, (n, self.Q, self.H)).astype(np.float32)
        s = np.zeros((n, self.Q, self.T), np.float32)
        idx = np.zeros((n, self.Q, self.TOPK), np.int32)
        for _ in range(min(warmup, 1)):
            cn.indexer(q, k, w, s, idx, self.H, nth)
        t0 = time.perf_counter()
        for _ in range(steps):
            cn.indexer(q, k, w, s, idx, self.H, nth)
        dt = time.perf_counter() - t0
        v = 2.0 * n * self.Q * self.H * self.D * self.T * steps / dt / 1e12
        return {"value": round(v, 6), "unit": "TFLOP/s", "steps": steps, "ms_per_step": round(dt / steps * 1e3, 3),
                "same_config": False, "cpu_baseline": {
                    "value": round(v, 6), "unit": "TFLOP/s", "cores": nth, "kind": "port",
                    "sample": f"1 of {self.B} batch elements per step (scoring + top-{self.TOPK}); C port of the "
                              f"indexer task bodies, {nth} threads"}}


class AttentionCase(Case):
    """Not a BASELINE config: the reference attention example's kernel at full tile sizes (f16 Q and K^T, f32 V and
    output, 128-row tiles), run by the fused tcgen05 kernel.  ``--workload attention``."""

    name, kernel, traffic_key = "attention", "attention_tile", ""
    unit, bound, dtype = "TFLOP/s", "tensor", "f16 Q.K^T / f32 softmax / W.V as 3 f16 terms / f32 out"
    metric = "attention-tile task-loop throughput (both contractions)"
    B, H, QT, L = 8, 16, 8, 1024

    def __init__(self, args):
        super().__init__(args)
        if args.batch:
            self.B = args.batch
        self.n_units = self.B

    @property
    def config(self) -> str:
        return (f"attention tiles {self.B}x{self.H}x{self.QT} (128 query rows each), {self.L} keys, d=128, "
                f"softmax(0.088 Q.K^T).V")

    def work(self) -> float:
        return 4.0 * self.B * self.H * self.QT * 128 * self.L * 128

    def plan(self):
        from pto_wsp_b200 import workloads

        return workloads.attention_plan(self.B, self.H, self.QT, self.L)

    def device_inputs(self, torch, dev):
        g = torch.Generator(device=dev)
        g.manual_seed(5000)
        q = torch.randn((self.B, self.H, self.QT, 128, 128), generator=g, device=dev).half()
        kt = torch.randn((self.B, self.H, 128, self.L), generator=g, device=dev).half()
        v = torch.randn((self.B, self.H, self.L, 128), generator=g, device=dev)
        o = torch.empty((self.B, self.H, self.QT, 128, 128), device=dev)
        return [q, kt, v, o]

    def check(self, darr) -> dict:
        torch = sys.modules["torch"]
        q, kt, v, o = darr
        s = torch.einsum("trd,dk->trk", q[0, 0].double(), kt[0, 0].double()) * float(np.float32(0.088))
        ref = torch.einsum("trk,kd->trd", torch.softmax(s, -1), v[0, 0].double())
        big = ref.abs() >= 1e-2 * ref.pow(2).mean().sqrt()
        return {"max_rel_err_vs_fp64_head0": float(((o[0, 0].double() - ref).abs() / ref.abs())[big].max())}

    def cpu_baseline(self, host, budget_s: float) -> dict:
        sys.path.insert(0, str(ROOT / "oracle"))
        from cpu_sim import CpuSim

        from pto_wsp_b200 import workloads

        sub = workloads.attention_plan(1, 1, 1, self.L)
        arrays = [np.ascontiguousarray(host[0][:1, :1, :1]), np.ascontiguousarray(host[1][:1, :1]),
                  np.ascontiguousarray(host[2][:1, :1]), np.zeros((1, 1, 1, 128, 128), np.float32)]
        t0 = time.perf_counter()
        CpuSim(sub).run(arrays)
        dt = time.perf_counter() - t0
        return {"value": round(4.0 * 128 * self.L * 128 / dt / 1e12, 7), "unit": "TFLOP/s", "cores": 1,
                "kind": "port", "sample": f"1 tile ({dt:.2f} s), numpy restatement of the tile program "
                                         f"(oracle/cpu_sim.py)"}

    def reference(self, steps: int, warmup: int) -> dict:
        b = self.cpu_baseline(workloads_attention_host(self), 0.0)
        return {"value": b["value"], "unit": "TFLOP/s", "steps": 1, "ms_per_step": None, "same_config": False,
                "cpu_baseline": b}


def workloads_attention_host(case: "AttentionCase"):
    rng = np.random.default_rng(5)
    return [rng.standard_normal((1, 1, 1, 128, 128)).astype(np.float16),
            rng.standard_normal((1, 1, 128, case.L)).astype(np.float16),
            rng.standard_normal((1, 1, case.L, 128)).astype(np.float32)]


CASES = {"softmax": SoftmaxCase, "rmsnorm": RmsNormCase, "bgemm": BgemmCase, "decode": DecodeCase,
         "indexer": IndexerCase, "attention": AttentionCase}


# ---------------------------------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------------------------------


class Dist:
    def __init__(self, world: int, local_rank: int):
        import torch

        self.torch = torch
        torch.cuda.set_device(local_rank)
        self.dev = torch.device("cuda", local_rank)
        self.local_rank = local_rank
        self.dist = None
        if world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=self.dev)
            self.dist = dist

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier(device_ids=[self.local_rank])
        self.torch.cuda.synchronize(self.dev)

    def max(self, v: float) -> float:
        if self.dist is None:
            return v
        t = self.torch.tensor([v], device=self.dev, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.dist is not None:
            self.dist.barrier(device_ids=[self.local_rank])
            self.dist.destroy_process_group()


def link_ceiling(D: Dist, h2d_bytes: int, d2h_bytes: int, reps: int = 3) -> dict:
    """The host link's floor for one end-to-end step: the time to copy the step's host->device bytes and its
    device->host bytes at once (pinned host buffers, one stream per direction, plain ``copy_``, best of ``reps``,
    max over ranks, which copy at the same time as they do in the timed steps).  ``frac`` of the ``e2e`` line is
    this floor over the measured step time."""
    torch, dev = D.torch, D.dev
    hin = torch.empty(max(h2d_bytes, 1), dtype=torch.uint8, pin_memory=True)
    hout = torch.empty(max(d2h_bytes, 1), dtype=torch.uint8, pin_memory=True)
    din = torch.empty(max(h2d_bytes, 1), dtype=torch.uint8, device=dev)
    dout = torch.zeros(max(d2h_bytes, 1), dtype=torch.uint8, device=dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    best = float("inf")
    for _ in range(reps):
        D.barrier()
        t0 = time.perf_counter()
        if h2d_bytes:
            with torch.cuda.stream(s_in):
                din.copy_(hin, non_blocking=True)
        if d2h_bytes:
            with torch.cuda.stream(s_out):
                hout.copy_(dout, non_blocking=True)
        torch.cuda.synchronize(dev)
        best = min(best, time.perf_counter() - t0)
    best = D.max(best)
    del hin, hout, din, dout
    return {"ms": round(best * 1e3, 3),
            "how": "the step's h2d and d2h bytes copied at once (pinned, one stream per direction, best of "
                   f"{reps}, max over ranks)"}


def run_case(case: Case, args, D: Dist, rank: int, world: int) -> dict:
    import numpy as np

    from pto_wsp_b200.shard import ShardedExecutable

    torch, dev = D.torch, D.dev
    plan = case.plan()
    darr = case.device_inputs(torch, dev)
    if args.partition:
        case.method = args.partition
    sh = ShardedExecutable(plan, rank=rank, world=world, device=D.local_rank, method=case.method,
                           costs=case.costs())
    units = sh.local_units(case.n_units)
    ex = sh.executable(len(units))
    stream = torch.cuda.current_stream(dev)
    ex.set_stream(stream)
    ex.set_option("sync", 0)
    axis = case.axis(case.n_units)

    def step(arrays):
        return sh.run_with_symbols(arrays, axis)

    for _ in range(args.warmup):
        step(darr)
    launches_per_step = int(ex.timing()["launches"])  # a replayed step launches the same kernels every time
    D.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with NvmlClockSampler(gpu_index(D.local_rank), _pci_bus_id(torch, dev)) as clk:
        # the timed region: K steps back to back, CUDA events on the launch stream around all of them
        D.barrier()
        h0 = time.perf_counter()
        e0.record(stream)
        for _ in range(args.steps):
            step(darr)
        e1.record(stream)
        host_ms = (time.perf_counter() - h0) * 1e3 / args.steps
        D.barrier()
        # the same K steps again with every kernel launch bracketed by CUDA events on the launch stream: the
        # dominant kernel's own launch time for the roofline (kept out of the pass above, whose steps the
        # extra event records would stretch)
        ex.set_option("kernel_events", 1)
        for _ in range(args.steps):
            step(darr)
        D.barrier()
        ktimes = ex.kernel_times()
        ex.set_option("kernel_events", 0)
    launches = launches_per_step * args.steps
    clocks = clk.summary()
    ms = e0.elapsed_time(e1)
    ms_max = D.max(ms)
    check = case.check(darr)

    # end to end: pinned host buffers through the same call, copies inside the timed region
    ex.set_option("sync", 1)
    if isinstance(case, BgemmCase):
        harr = case.host_views(torch)
    else:
        harr = []
        for t in darr:
            h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            h.copy_(t)
            harr.append(h.numpy())
    step(harr)  # device staging buffers and layout checks
    e2e_steps = args.e2e_steps or min(args.steps, 10)
    D.barrier()
    t0 = time.perf_counter()
    h2d = d2h = 0
    for _ in range(e2e_steps):
        step(harr)
        tm = ex.timing()
        h2d += tm["h2d_bytes"]
        d2h += tm["d2h_bytes"]
    D.barrier()
    e2e_s = D.max(time.perf_counter() - t0)
    link = link_ceiling(D, h2d // e2e_steps, d2h // e2e_steps)
    link["e2e_ms"] = round(e2e_s * 1e3 / e2e_steps, 3)
    link["frac"] = round(link["ms"] / link["e2e_ms"], 4) if link["e2e_ms"] > 0 else None

    work = case.work()
    value = work * args.steps / (ms_max / 1e3) / case.scale
    e2e = work * e2e_steps / e2e_s / case.scale
    peak, peak_kind = peaks("hbm_gbs" if case.bound == "hbm" else "bf16_tflops")
    kt = ktimes.get(case.kernel, {"launches": 0, "ms": 0.0})
    kwork = case.unit_work(units)
    per_launch_ms = kt["ms"] / max(kt["launches"], 1)
    achieved = kwork / (per_launch_ms / 1e3) / case.scale if per_launch_ms > 0 else 0.0
    traffic = traffic_from_profiles(case.traffic_key)
    if traffic is not None and not args.batch and not args.cols:
        traffic = traffic * kwork / case.unit_work(list(range(case.n_units)))
    else:
        traffic = None
    line = {
        "metric": case.metric, "value": round(value, 3), "unit": case.unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": case.dtype,
        "data": "synthetic (seeded torch generators on device; BASELINE.json shapes and distributions)",
        "config": {"workload": case.config, "global_batch": case.n_units, "rank_units": len(units),
                   "parallelism": f"P(batch) over {world} rank(s), {case.method} shares (ShardedExecutable)",
                   "l2": "every step reads inputs larger than the 126 MB L2 (no flush)"},
        "gpu_launches": launches,
        "host_ms_per_step": round(host_ms, 4),
        "roofline": {"bound": case.bound, "achieved": round(achieved, 2), "peak": peak, "unit": case.unit,
                     "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                     "kernel": case.kernel,
                     ("bytes_per_launch" if case.bound == "hbm" else "flops_per_launch"): kwork,
                     "launch_ms": round(per_launch_ms, 5), "launches_timed": kt["launches"],
                     "timing": "CUDA events around each of the kernel's launches on the launch stream, over a second "
                               "pass of the K timed steps"},
        "kernel_ms": {k: {"launches": v["launches"], "ms_per_launch": round(v["ms"] / max(v["launches"], 1), 5)}
                      for k, v in ktimes.items()},
        "e2e": {"value": round(e2e, 4), "unit": case.unit, "h2d_bytes_per_step": h2d // e2e_steps,
                "d2h_bytes_per_step": d2h // e2e_steps, "steps": e2e_steps,
                "path": "ShardedExecutable.run_with_symbols (CodegenExecutable surface) with pinned numpy buffers",
                "link": link},
        "clocks": clocks,
        "check": check,
    }
    if case.bound == "tensor":
        line["roofline"]["peak_kind"] += " (cuBLAS bf16 burst; f16 runs at the same tensor rate)"
    if isinstance(case, IndexerCase):
        step_ach = case.unit_work(units) / (ms / args.steps / 1e3) / 1e12
        line["roofline"]["step_frac"] = round(step_ach / peak, 4)
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = case.cpu_baseline(harr, args.cpu_budget)
    del darr, harr
    torch.cuda.empty_cache()
    return line


def run_gpu(args, names: list[str], rank: int, world: int, local_rank: int) -> None:
    D = Dist(world, local_rank)
    lines = {}
    for n in names:
        lines[n] = run_case(CASES[n](args), args, D, rank, world)
    if rank == 0:
        head = dict(lines[names[0]])
        if len(names) > 1:
            head["workloads"] = {n: lines[n] for n in names[1:]}
        print(json.dumps(head), flush=True)
    D.close()


def artifact_units(case: Case, procs: int) -> tuple[list[dict], str, bool] | None:
    """The units of one reference step (each one artifact call), what they are, and whether they are the whole
    config; None when the built artifact does not have this case's unit shape."""
    if case.args.batch or case.args.cols:
        return None
    if isinstance(case, RowCase):
        return [{"index": i} for i in range(case.batch)], f"the whole config ({case.batch} batch elements)", True
    if isinstance(case, BgemmCase):
        n = min(procs, case.B * case.M // 128)
        return ([{"index": i} for i in range(n)],
                f"{n} of the config's {case.B * case.M // 128} 128-row slabs (one per process)", False)
    if isinstance(case, DecodeCase):
        return ([{"index": r, "length": int(case.lens[r])} for r in range(case.R)],
                f"the whole config ({case.R} requests, the bench's KV lengths)", True)
    if isinstance(case, IndexerCase):
        n = min(procs, case.B)
        return [{"index": i} for i in range(n)], f"{n} of the config's {case.B} batch elements", n == case.B
    return None


def unit_work(case: Case, unit: dict) -> float:
    if isinstance(case, RowCase):
        return case.tiles * case.rows * case.cols * 8.0
    if isinstance(case, BgemmCase):
        return 2.0 * 128 * case.N * case.K
    if isinstance(case, DecodeCase):
        return case.unit_work([unit["index"]])
    return case.work() / case.B


def reference_artifact(case: Case, args, budget_s: float = 20.0) -> dict | None:
    """The reference's own CPU-sim artifact of this config (oracle/_ref), one process per host core."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import ref_runner

    if ref_runner.manifest() is None:
        return None
    procs = ref_runner.host_cores()
    spec = artifact_units(case, procs)
    if spec is None:
        return None
    units, what, whole = spec
    work = sum(unit_work(case, u) for u in units)
    pool = ref_runner.Pool(case.name, units, procs, seed=7)
    try:
        warm = [pool.step()[0]]  # one warm-up step: the artifact has nothing to compile, this pages it in
        steps = max(1, min(args.steps, int(budget_s / max(min(warm), 1e-3))))
        busy = 0.0
        t0 = time.perf_counter()
        for _ in range(steps):
            busy += sum(pool.step()[1])
        dt = time.perf_counter() - t0
    finally:
        pool.close()
    v = work * steps / dt / case.scale
    one_core = work * steps / busy / case.scale
    sample = (f"{what} per step; the reference's own CPU-sim artifact (its generated task loop and kernels, built "
              f"with the clean-room pto-isa stand-in) through its CodegenExecutable, {pool.procs} processes "
              f"(single-threaded each, as the CPU-sim is); 1-core rate {one_core:.6g} {case.unit}")
    return {"value": round(v, 6), "unit": case.unit, "steps": steps, "ms_per_step": round(dt / steps * 1e3, 3),
            "same_config": whole, "single_core": round(one_core, 6),
            "cpu_baseline": {"value": round(v, 6), "unit": case.unit, "cores": pool.procs, "kind": "reference",
                             "sample": sample}}


def run_reference(args, names: list[str], rank: int) -> None:
    if rank != 0:
        return
    lines = {}
    for n in names:
        case = CASES[n](args)
        r = reference_artifact(case, args) or case.reference(args.steps, args.warmup)
        lines[n] = {"impl": "reference", "metric": case.metric, "value": r["value"], "unit": r["unit"],
                    "n_gpus": args.gpus, "steps": r["steps"], "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
                    "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": case.dtype,
                    "data": "synthetic (seeded numpy)", "config": {"workload": case.config,
                                                                   "same_config": r["same_config"]},
                    "cpu_baseline": r["cpu_baseline"],
                    "e2e": {"value": r["value"], "unit": r["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        if "single_core" in r:
            lines[n]["single_core"] = {"value": r["single_core"], "unit": r["unit"], "cores": 1}
    head = dict(lines[names[0]])
    if len(names) > 1:
        head["workloads"] = {n: lines[n] for n in names[1:]}
    print(json.dumps(head), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="all", choices=["all"] + ORDER + ["attention"])
    ap.add_argument("--e2e-steps", type=int, default=None, help="steps of the end-to-end leg (default min(steps, 10))")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=4.0, help="seconds of CPU work per cpu_baseline sample")
    ap.add_argument("--batch", type=int, default=None, help="override the outer batch (small profiling cases)")
    ap.add_argument("--partition", default=None, choices=["block", "balanced", "lpt"],
                    help="override the workloads' share method over the ranks")
    ap.add_argument("--cols", type=int, default=None, help="rmsnorm/softmax: another tile width (row-program kernel)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    names = ORDER if args.workload == "all" else [args.workload]
    rank, world, local_rank = _env_int("RANK", 0), _env_int("WORLD_SIZE", 1), _env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        run_reference(args, names, rank)
    else:
        run_gpu(args, names, rank, world, local_rank)


if __name__ == "__main__":
    main()
