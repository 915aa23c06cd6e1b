#!/usr/bin/env python3
"""Benchmark of the PTO-WSP cuda_sm100a task loop (one JSON line on rank 0).

Default workload: BASELINE config 2, the row-softmax tile workload
X[32,2048,32,256] f32 (Tile[32,256], P(batch) x P(tiles)), through the
reference-facing C ABI.  A *step* is one pass of the task loop over the whole
workload.

* ``value``  -- GB/s (algorithmic bytes: 2 x 4 B per element) with X and Y
  resident in HBM; K back-to-back steps timed with CUDA events on the launch
  stream, max over ranks.  Inputs (2 GiB) exceed L2 (126 MB), so no flush.
* ``e2e``    -- the same metric through the same call with pinned host numpy
  buffers: every step stages X host->device and Y device->host.
* ``roofline`` -- achieved bytes per launch / measured launch time vs the
  measured HBM copy peak (MEASURED_PEAKS.json); ``traffic`` from the ncu
  summary in profiles/ when one exists.
* ``cpu_baseline`` -- the C port of the CPU-sim loops (oracle/cpu_kernels.c) on
  the host cores, rank 0 at N=1, bounded sample.

``--impl reference`` times only that CPU implementation (all host threads) and
prints its own line.  Multi-GPU (torchrun): each rank runs the same per-rank
shard (weak scaling, no data-path collective).
"""

from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import threading
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    "softmax": {"config": "config 2: row softmax Tile[32,256] f32, X[32,2048,32,256]", "batch": 32, "tiles": 2048,
                "rows": 32, "cols": 256},
    "rmsnorm": {"config": "config 1: RMSNorm Tile[16,128] f32, X[64,4096,16,128] (GPU scale)", "batch": 64,
                "tiles": 4096, "rows": 16, "cols": 128},
    "bgemm": {"config": "config 3: bgemm 64 x (2048x2048x2048), f16 in, f32 acc/out, 128x128 output tiles",
              "batch": 64, "m": 2048, "n": 2048, "k": 2048},
    "decode": {"config": "config 4: paged GQA decode, 64 requests, 32 q / 8 kv heads, d=128, f16, page 16, "
                         "KV len U[512,8192]", "batch": 64},
    "indexer": {"config": "config 5: lightning indexer 16 batches x 8 queries, 64 heads, d=128, 32768 keys, "
                          "top-2048", "batch": 16, "context": 32768, "topk": 2048},
}


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


def traffic_from_profiles(kernel: str, workload: str, batch_override=None) -> float | None:
    """DRAM bytes per launch of the full workload from the committed ncu summaries (None for --batch runs)."""
    p = ROOT / "profiles" / "traffic.json"
    if batch_override is not None or not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        v = d.get(f"{workload}:{kernel}")
        return float(v["bytes_per_launch"]) if v else None
    except Exception:  # noqa: BLE001
        return None


class NvmlClockSampler:
    """SM clock, power and clock-event reasons read through NVML every millisecond while the timed region runs
    (read-only queries; short timed regions still get several samples).  Falls back to nvidia-smi."""

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
    """The NVML-style PCI bus id of a torch CUDA device, when torch exposes it."""
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


def make_softmax_inputs(torch, B, T, R, Cc, device, seed=0):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn((B, T, R, Cc), generator=g, device=device, dtype=torch.float32) * 4.0
    mask = torch.rand((B, T, R, Cc), generator=g, device=device) < 0.01
    x[mask] = 30.0
    return x


def make_rmsnorm_inputs(torch, B, T, R, Cc, device, seed=0):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn((B, T, R, Cc), generator=g, device=device, dtype=torch.float32)


def cpu_baseline(kind: str, x_host, rows: int, cols: int, budget_s: float = 12.0) -> dict:
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np

    import cpu_native

    nth = cpu_native.threads()
    tiles_total = x_host.size // (rows * cols)
    flat = x_host.reshape(tiles_total, rows, cols)
    n = min(tiles_total, 2048)
    y = np.empty_like(flat[:n])
    t0 = time.perf_counter()
    cpu_native.row_tiles(kind, np.ascontiguousarray(flat[:n]), y, rows, cols, nth)
    dt = time.perf_counter() - t0
    # grow the sample to ~budget_s of CPU work (bounded by the workload)
    n2 = int(min(tiles_total, max(n, n * budget_s / max(dt, 1e-6) * 0.5)))
    passes = max(1, min(8, int(budget_s / max(dt * n2 / n, 1e-6))))
    y = np.empty((n2, rows, cols), np.float32)
    t0 = time.perf_counter()
    for _ in range(passes):
        cpu_native.row_tiles(kind, flat[:n2], y, rows, cols, nth)
    dt = time.perf_counter() - t0
    gbs = passes * n2 * rows * cols * 8 / dt / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": nth, "kind": "port",
            "sample": f"{passes} pass(es) over {n2} of {tiles_total} tiles ({n2 * rows * cols * 4 / 2**20:.0f} MiB in), "
                      f"{dt:.2f} s, C port of the CPU-sim tile loop (oracle/cpu_kernels.c), {nth} threads"}


def run_reference(args, wl: dict, rank: int) -> None:
    if rank != 0:
        return
    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    import cpu_native

    rows, cols = wl["rows"], wl["cols"]
    tiles = wl["batch"] * wl["tiles"]
    sample_tiles = min(tiles, 8192)
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((sample_tiles, rows, cols), dtype=np.float32) * (4.0 if args.workload == "softmax" else 1.0))
    if args.workload == "softmax":
        x[rng.random(x.shape) < 0.01] = 30.0
    y = np.empty_like(x)
    nth = cpu_native.threads()
    for _ in range(args.warmup):
        cpu_native.row_tiles(args.workload, x, y, rows, cols, nth)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_native.row_tiles(args.workload, x, y, rows, cols, nth)
    dt = time.perf_counter() - t0
    gbs = sample_tiles * rows * cols * 8 * args.steps / dt / 1e9
    line = {
        "impl": "reference", "metric": f"{args.workload} task-loop throughput (algorithmic HBM bytes)",
        "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded numpy)",
        "config": {"workload": wl["config"], "sample_tiles_per_step": sample_tiles},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": nth, "kind": "port",
                         "sample": f"{sample_tiles} tiles per step of {tiles}; C port of the CPU-sim tile loop "
                                   f"(oracle/cpu_kernels.c), {nth} threads (reference CPU-sim needs the absent pto-isa)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def gemm_cpu_baseline(a_host, b_host, tiles: int = 128, budget_s: float = 10.0) -> dict:
    """C port of the CPU-sim gemm task (TLOAD, TMATMUL f32 acc, TSTORE) on a bounded batch sample."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np

    import cpu_native

    nth = cpu_native.threads()
    B, M, K = a_host.shape
    N = b_host.shape[2]
    nb = 1
    t0 = time.perf_counter()
    c = np.empty((nb, M, N), np.float32)
    cpu_native.gemm_tiles(a_host[:nb], b_host[:nb], c, tiles, tiles, nth)
    dt = time.perf_counter() - t0
    nb2 = int(max(1, min(B, budget_s / max(dt, 1e-6))))
    if nb2 > 1:
        c = np.empty((nb2, M, N), np.float32)
        t0 = time.perf_counter()
        cpu_native.gemm_tiles(a_host[:nb2], b_host[:nb2], c, tiles, tiles, nth)
        dt = time.perf_counter() - t0
    else:
        nb2 = nb
    tf = 2.0 * nb2 * M * N * K / dt / 1e12
    return {"value": round(tf, 5), "unit": "TFLOP/s", "cores": nth, "kind": "port",
            "sample": f"{nb2} of {B} batch elements ({dt:.2f} s), C port of the CPU-sim gemm tile task "
                      f"(oracle/cpu_kernels.c, f32 accumulation), {nth} threads"}


def run_bgemm(args, wl: dict, rank: int, world: int, local_rank: int) -> None:
    B, M, N, K = wl["batch"], wl["m"], wl["n"], wl["k"]
    flops = 2.0 * B * M * N * K
    if args.impl == "reference":
        if rank != 0:
            return
        import numpy as np

        sys.path.insert(0, str(ROOT / "oracle"))
        import cpu_native

        rng = np.random.default_rng(0)
        nb = 1
        a = rng.uniform(-1, 1, (nb, M, K)).astype(np.float16)
        b = rng.uniform(-1, 1, (nb, K, N)).astype(np.float16)
        c = np.empty((nb, M, N), np.float32)
        nth = cpu_native.threads()
        # bounded step: a 512-row slab of one batch element per step
        rows = 512
        for _ in range(args.warmup):
            cpu_native.gemm_tiles(a[:, :rows], b, c[:, :rows], 128, 128, nth)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            cpu_native.gemm_tiles(a[:, :rows], b, c[:, :rows], 128, 128, nth)
        dt = time.perf_counter() - t0
        tf = 2.0 * rows * N * K * args.steps / dt / 1e12
        print(json.dumps({
            "impl": "reference", "metric": "bgemm task-loop throughput", "value": round(tf, 5), "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 in / f32 acc", "data": "synthetic (seeded numpy)",
            "config": {"workload": wl["config"], "sample_per_step": f"{rows}x{N}x{K} slab of one batch element"},
            "cpu_baseline": {"value": round(tf, 5), "unit": "TFLOP/s", "cores": nth, "kind": "port",
                             "sample": f"{rows}-row slab per step; C port of the CPU-sim gemm task, {nth} threads"},
            "e2e": {"value": round(tf, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return

    import numpy as np
    import torch

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    from pto_wsp_b200 import workloads
    from pto_wsp_b200.runtime import CudaExecutable

    g = torch.Generator(device=dev)
    g.manual_seed(2000 + rank)
    a = (torch.rand((B, M, K), generator=g, device=dev) * 2 - 1).half()
    b = (torch.rand((B, K, N), generator=g, device=dev) * 2 - 1).half()
    c = torch.empty((B, M, N), device=dev, dtype=torch.float32)
    ex = CudaExecutable(workloads.bgemm_plan(B, M, N, K), device=local_rank)
    stream = torch.cuda.current_stream(dev)
    ex.set_stream(stream)
    ex.set_option("sync", 0)
    views = list(workloads.bgemm_views(a, b, c))

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        ex.run_with_symbols(views, {}, {}, {})
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    with NvmlClockSampler(gpu_index(local_rank), _pci_bus_id(torch, dev)) as clk:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            ex.run_with_symbols(views, {}, {}, {})
            launches += int(ex.timing()["launches"])
        e1.record(stream)
        barrier()
        ms = e0.elapsed_time(e1)
        ms_max = max_over_ranks(ms)
        # end to end with pinned host buffers
        ex.set_option("sync", 1)
        ah_t = torch.empty(a.shape, dtype=a.dtype, pin_memory=True)
        bh_t = torch.empty(b.shape, dtype=b.dtype, pin_memory=True)
        ch_t = torch.empty(c.shape, dtype=c.dtype, pin_memory=True)
        ah_t.copy_(a)
        bh_t.copy_(b)
        ah, bh, ch = ah_t.numpy(), bh_t.numpy(), ch_t.numpy()
        hviews = list(workloads.bgemm_views(ah, bh, ch))
        ex.run_with_symbols(hviews, {}, {}, {})
        e2e_steps = args.e2e_steps or min(args.steps, 10)
        barrier()
        t0 = time.perf_counter()
        h2d = d2h = 0
        for _ in range(e2e_steps):
            ex.run_with_symbols(hviews, {}, {}, {})
            tm = ex.timing()
            h2d += tm["h2d_bytes"]
            d2h += tm["d2h_bytes"]
        barrier()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
    clocks = clk.summary()
    value = world * flops * args.steps / (ms_max / 1e3) / 1e12
    e2e = world * flops * e2e_steps / e2e_s / 1e12
    peak, peak_kind = peaks("bf16_tflops")
    achieved = flops / (ms / args.steps / 1e3) / 1e12
    ref = (a[0].double() @ b[0].double())
    err = float(((c[0].double() - ref).abs() / (ref.abs() + ref.pow(2).mean().sqrt())).max())
    if rank == 0:
        line = {
            "metric": "bgemm task-loop throughput", "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16 in / f32 acc",
            "data": "synthetic (seeded torch.rand on device, U(-1,1))",
            "config": {"workload": wl["config"], "global_batch": B * world, "per_rank_batch": B,
                       "parallelism": f"P(batch) sharded, {world} rank(s)",
                       "l2": "operands 1 GiB > 126 MB L2 (no flush needed)"},
            "gpu_launches": launches,
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic_from_profiles("matmul_tcgen05", "bgemm", args.batch),
                         "peak_kind": peak_kind + " (cuBLAS bf16 burst; fp16 runs at the same tensor rate)",
                         "kernel": "matmul_tcgen05", "flops_per_launch": flops},
            "e2e": {"value": round(e2e, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d // e2e_steps,
                    "d2h_bytes_per_step": d2h // e2e_steps, "steps": e2e_steps},
            "clocks": clocks,
            "max_rel_err_vs_fp64_batch0": err,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = gemm_cpu_baseline(ah, bh)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def _dist_setup(world: int, local_rank: int):
    import torch

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    return torch, dev, dist


def run_builtin(args, wl: dict, rank: int, world: int, local_rank: int) -> None:
    """Configs 4 (paged decode, GB/s) and 5 (indexer scoring + top-k, TFLOP/s of the scoring)."""
    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    if args.impl == "reference":
        if rank != 0:
            return
        from cpu_sim import CpuSim

        from pto_wsp_b200 import workloads

        rng = np.random.default_rng(0)
        if args.workload == "decode":
            plan, arrays = workloads.decode_inputs(rng, 4)  # bounded sample: 4 requests x 8 kv heads per step
            unit_bytes = int(arrays[4].astype(np.int64).sum()) * 8 * 128 * 2 * 2
            work, unit = unit_bytes, "GB/s"
            axis = {"b": 4}
        else:
            plan, arrays = workloads.indexer_inputs(rng, 1, wl["context"], wl["topk"])
            work, unit = 2.0 * 512 * 128 * wl["context"], "TFLOP/s"
            axis = {}
        sim = CpuSim(plan)
        for _ in range(min(args.warmup, 1)):
            sim.run([a.copy() for a in arrays], axis_sizes=axis)
        steps = max(1, min(args.steps, 5))
        t0 = time.perf_counter()
        for _ in range(steps):
            sim.run([a.copy() for a in arrays], axis_sizes=axis)
        dt = time.perf_counter() - t0
        v = work * steps / dt / (1e9 if unit == "GB/s" else 1e12)
        sample = ("4 requests x 8 kv heads per step" if args.workload == "decode" else "1 batch element per step")
        print(json.dumps({
            "impl": "reference", "metric": f"{args.workload} task-loop throughput", "value": round(v, 5), "unit": unit,
            "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup, "ms_per_step": round(dt / steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16 in / f32",
            "data": "synthetic (seeded numpy)", "config": {"workload": wl["config"], "sample_per_step": sample},
            "cpu_baseline": {"value": round(v, 5), "unit": unit, "cores": 1, "kind": "port",
                             "sample": sample + "; numpy restatement of the CPU-sim task (oracle/cpu_sim.py)"},
            "e2e": {"value": round(v, 5), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return

    torch, dev, dist = _dist_setup(world, local_rank)
    from pto_wsp_b200 import workloads
    from pto_wsp_b200.runtime import CudaExecutable

    rng = np.random.default_rng(3000 + rank)
    if args.workload == "decode":
        R = wl["batch"]
        plan, host = workloads.decode_inputs(rng, R)
        lens = host[4].astype(np.int64).reshape(-1)
        work = float(lens.sum() * 8 * 128 * 2 * 2 + R * 32 * 128 * 2 * 2)  # K+V of every token + Q + O
        unit, scale, kname, bound = "GB/s", 1e9, "paged_decode_tma", "hbm"
        axis = {"b": R}
    else:
        B, T, K = wl["batch"], wl["context"], wl["topk"]
        plan, host = workloads.indexer_inputs(rng, B, T, K)
        work = 2.0 * B * 512 * 128 * T
        unit, scale, kname, bound = "TFLOP/s", 1e12, "indexer_score", "tensor"
        axis = {}
    ex = CudaExecutable(plan, device=local_rank)
    stream = torch.cuda.current_stream(dev)
    ex.set_stream(stream)
    ex.set_option("sync", 0)
    darr = [torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in host]

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        ex.run_with_symbols(darr, axis, {}, {})
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    with NvmlClockSampler(gpu_index(local_rank), _pci_bus_id(torch, dev)) as clk:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            ex.run_with_symbols(darr, axis, {}, {})
            launches += int(ex.timing()["launches"])
        e1.record(stream)
        barrier()
        ms = e0.elapsed_time(e1)
        ms_max = max_over_ranks(ms)
        ex.set_option("sync", 1)
        pinned = []
        for a in host:
            t = torch.empty(a.shape, dtype=torch.from_numpy(a[:0].copy()).dtype, pin_memory=True)
            t.copy_(torch.from_numpy(np.ascontiguousarray(a)))
            pinned.append(t.numpy())
        ex.run_with_symbols(pinned, axis, {}, {})
        e2e_steps = args.e2e_steps or min(args.steps, 10)
        barrier()
        t0 = time.perf_counter()
        h2d = d2h = 0
        for _ in range(e2e_steps):
            ex.run_with_symbols(pinned, axis, {}, {})
            tm = ex.timing()
            h2d += tm["h2d_bytes"]
            d2h += tm["d2h_bytes"]
        barrier()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
    clocks = clk.summary()
    value = world * work * args.steps / (ms_max / 1e3) / scale
    e2e = world * work * e2e_steps / e2e_s / scale
    peak, peak_kind = peaks("hbm_gbs" if bound == "hbm" else "bf16_tflops")
    achieved = work / (ms / args.steps / 1e3) / scale
    if rank == 0:
        line = {
            "metric": f"{args.workload} task-loop throughput", "value": round(value, 3), "unit": unit,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16 in / f32 softmax|acc",
            "data": "synthetic (seeded numpy, BASELINE.json distributions)",
            "config": {"workload": wl["config"], "per_rank_batch": wl["batch"], "global_batch": wl["batch"] * world,
                       "parallelism": f"P(batch) sharded, {world} rank(s)",
                       "l2": "KV / keys > 126 MB L2 (no flush needed)"},
            "gpu_launches": launches,
            "roofline": {"bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
                         "frac": round(achieved / peak, 4), "traffic": traffic_from_profiles(kname, args.workload, args.batch),
                         "peak_kind": peak_kind, "kernel": kname,
                         ("bytes_per_launch" if bound == "hbm" else "flops_per_launch"): work,
                         "note": "step = all work of the task loop (decode: counter memset + TMA kernel with fused merge; indexer: scoring + "
                                 "top-k); achieved uses the whole step time"},
            "e2e": {"value": round(e2e, 4), "unit": unit, "h2d_bytes_per_step": h2d // e2e_steps,
                    "d2h_bytes_per_step": d2h // e2e_steps, "steps": e2e_steps},
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            from cpu_sim import CpuSim

            if args.workload == "decode":
                sub_plan, sub = workloads.decode_inputs(np.random.default_rng(1), 2)
                sub_work = float(sub[4].astype(np.int64).sum() * 8 * 128 * 2 * 2)
                ax = {"b": 2}
                what = "2 requests x 8 kv heads"
            else:
                sub_plan, sub = workloads.indexer_inputs(np.random.default_rng(1), 1, wl["context"], wl["topk"])
                sub_work = 2.0 * 512 * 128 * wl["context"]
                ax = {}
                what = "1 batch element (scoring + top-k)"
            t0 = time.perf_counter()
            CpuSim(sub_plan).run(sub, axis_sizes=ax)
            dt = time.perf_counter() - t0
            line["cpu_baseline"] = {"value": round(sub_work / dt / scale, 6), "unit": unit, "cores": 1,
                                    "kind": "port", "sample": f"{what}, {dt:.2f} s, numpy restatement of the "
                                                              f"CPU-sim task (oracle/cpu_sim.py)"}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="softmax", choices=sorted(WORKLOADS))
    ap.add_argument("--e2e-steps", type=int, default=None, help="steps of the end-to-end leg (default: --steps, max 20)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None, help="override the per-rank batch (small profiling cases)")
    ap.add_argument("--cols", type=int, default=None,
                    help="rmsnorm/softmax: tile width other than the config's (widths without a hand-written row "
                         "kernel run the fused row-program kernel built at run time)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    wl = dict(WORKLOADS[args.workload])
    if args.batch:
        wl["batch"] = args.batch
        wl["config"] += f" [batch overridden to {args.batch}]"
    if args.cols and "cols" in wl:
        wl["cols"] = args.cols
        wl["config"] += f" [tile width overridden to {args.cols}]"

    rank = _env_int("RANK", 0)
    world = _env_int("WORLD_SIZE", 1)
    local_rank = _env_int("LOCAL_RANK", 0)

    if args.workload == "bgemm":
        run_bgemm(args, wl, rank, world, local_rank)
        return
    if args.workload in ("decode", "indexer"):
        run_builtin(args, wl, rank, world, local_rank)
        return
    if args.impl == "reference":
        run_reference(args, wl, rank)
        return

    import numpy as np
    import torch

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    from pto_wsp_b200 import workloads
    from pto_wsp_b200.runtime import CudaExecutable

    B, T, R, Cc = wl["batch"], wl["tiles"], wl["rows"], wl["cols"]
    plan = (workloads.softmax_plan if args.workload == "softmax" else workloads.rmsnorm_plan)(B, T, R, Cc)
    ex = CudaExecutable(plan, device=local_rank)
    stream = torch.cuda.current_stream(dev)
    ex.set_stream(stream)
    ex.set_option("sync", 0)
    mk = make_softmax_inputs if args.workload == "softmax" else make_rmsnorm_inputs
    x = mk(torch, B, T, R, Cc, dev, seed=1000 + rank)
    y = torch.empty_like(x)
    elems = x.numel()
    alg_bytes = elems * 8  # read x + write y, f32

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident value ----
    for _ in range(args.warmup):
        ex.run_with_symbols([x, y], {}, {}, {})
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    with NvmlClockSampler(gpu_index(local_rank), _pci_bus_id(torch, dev)) as clk:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            ex.run_with_symbols([x, y], {}, {}, {})
            launches += int(ex.timing()["launches"])
        e1.record(stream)
        barrier()
        ms = e0.elapsed_time(e1)
        ms_max = max_over_ranks(ms)

        # ---- end-to-end through the same call with pinned host buffers ----
        ex.set_option("sync", 1)
        xh_t = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        yh_t = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        xh_t.copy_(x)
        xh, yh = xh_t.numpy(), yh_t.numpy()
        e2e_steps = args.e2e_steps or min(args.steps, 20)
        ex.run_with_symbols([xh, yh], {}, {}, {})  # warm: device staging buffers
        barrier()
        t0 = time.perf_counter()
        h2d = d2h = 0
        for _ in range(e2e_steps):
            ex.run_with_symbols([xh, yh], {}, {}, {})
            tm = ex.timing()
            h2d += tm["h2d_bytes"]
            d2h += tm["d2h_bytes"]
        barrier()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
    clocks = clk.summary()

    value = world * alg_bytes * args.steps / (ms_max / 1e3) / 1e9
    e2e = world * alg_bytes * e2e_steps / e2e_s / 1e9
    peak, peak_kind = peaks()
    per_launch_ms = ms / args.steps
    achieved = alg_bytes / (per_launch_ms / 1e3) / 1e9
    kernel_name = "softmax_rows" if args.workload == "softmax" else "rmsnorm_rows"
    if ex.describe()["kernels"][0].get("row_kernel") == "loaded":
        kernel_name = "ptowsp_rows_k0 (row program built with NVRTC)"
    traffic = traffic_from_profiles(kernel_name, args.workload, args.batch or args.cols)

    # spot-check the last device result against the numpy definition on a few tiles
    xs = x.reshape(-1, R, Cc)[:64].double().cpu().numpy()
    ys = y.reshape(-1, R, Cc)[:64].double().cpu().numpy()
    if args.workload == "softmax":
        ref = np.exp(xs - xs.max(-1, keepdims=True))
        ref /= ref.sum(-1, keepdims=True)
    else:
        ref = xs / np.sqrt((xs * xs).mean(-1, keepdims=True))
    check = float(np.max(np.abs(ys - ref) / (np.abs(ref) + 1e-30)))

    if rank == 0:
        line = {
            "metric": f"{args.workload} task-loop throughput (algorithmic HBM bytes)",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded torch.randn on device)",
            "config": {"workload": wl["config"], "global_batch": B * world, "per_rank_batch": B, "tiles": T,
                       "tile": [R, Cc], "parallelism": f"P(batch) sharded, {world} rank(s)",
                       "l2": "inputs 2 GiB > 126 MB L2 (no flush needed)"},
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                         "kernel": kernel_name, "bytes_per_launch": alg_bytes},
            "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d // e2e_steps,
                    "d2h_bytes_per_step": d2h // e2e_steps, "steps": e2e_steps,
                    "path": "CodegenExecutable-style run_with_symbols with pinned numpy buffers"},
            "clocks": clocks,
            "max_rel_err_vs_fp64_sample": check,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.workload, xh, R, Cc)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
