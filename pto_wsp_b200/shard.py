"""Sharding a plan's outermost ``P(batch)`` axis over the GPUs of one node.

Every unit of a workload's outermost ``ParallelFor`` is independent of the
others -- RMSNorm/softmax tiles of a batch element, a bgemm batch, a decode
request, an indexer batch -- because the reference emits the loop nest as
plain nested loops whose bodies only index their own slice
(``src/python/pto_codegen.cpp:2305-2360``).  So a rank runs the *same* plan
over its share of the units, one process per GPU, with no data-path
collective:

* the partition is contiguous blocks (configs 1, 2, 3, 5) or a greedy
  longest-processing-time assignment by a per-unit cost (config 4's requests,
  whose KV lengths differ 16x);
* tensors indexed by the outer loop variable in their first dimension are
  sliced to the rank's units (zero-copy views for a contiguous block, gathered
  copies otherwise, scattered back after the run); every other tensor is read
  whole by every rank and must not be written;
* where a tensor's layout is replicated while the computation is
  batch-sharded (``TensorLayout.default`` vs ``TensorLayout.sharded(0, ...)``,
  reference ``python/pto_wsp/types.py:285-294``), its shards are gathered over
  the ranks after the run -- the ``relayout`` / ``allgather`` step of
  ``python/pto_wsp/types.py:539-615`` -- through ``torch.distributed``
  (NCCL over NVLink for CUDA tensors and NCCL groups, gloo for host tensors).
  The gather is timed separately from the kernels.

The per-rank executable is a :class:`~pto_wsp_b200.runtime.CudaExecutable`
compiled from the rank's plan (outer axis size and sharded tensor shapes set
to the rank's unit count).
"""

from __future__ import annotations

import copy
import os
import time
from typing import Any, Callable, Sequence


class ShardError(ValueError):
    """The plan's loop nest cannot be split over its outermost axis."""


# ---------------------------------------------------------------------------
# Plan analysis
# ---------------------------------------------------------------------------


def outer_loops(plan: dict) -> list[dict]:
    """The outermost parallel loops: the body itself, or every child of a top-level combine / sequential."""
    body = plan["body"]
    if body.get("kind") == "parallel_for":
        return [body]
    if body.get("kind") in ("combine", "sequential"):
        kids = body.get("children", [])
        if kids and all(k.get("kind") == "parallel_for" for k in kids):
            return list(kids)
    raise ShardError("the workload's outermost node is not a P() loop (or a combination of P() loops)")


def _outer_size(loops: list[dict]) -> int | None:
    sizes = set()
    for lp in loops:
        ax = lp["axis"]
        if ax["kind"] == "dense":
            sizes.add(int(ax["size"]))
        elif ax["kind"] == "dense_dyn":
            sizes.add(None)
        else:
            raise ShardError(f"outer axis kind {ax['kind']!r} cannot be sharded (dense / dense_dyn only)")
    if len(sizes) != 1:
        raise ShardError("the outer P() loops of the workload have different sizes")
    return sizes.pop()


def _walk(node: dict, fn: Callable[[dict], None]) -> None:
    """Call `fn` on `node` and every workload node below it."""
    fn(node)
    for key in ("body", "then", "else"):
        if isinstance(node.get(key), dict):
            _walk(node[key], fn)
    for c in node.get("children", []) or []:
        _walk(c, fn)


def _mentions(expr: Any, var: str) -> bool:
    if isinstance(expr, dict):
        return expr.get("var") == var or any(_mentions(v, var) for v in expr.values())
    if isinstance(expr, list):
        return any(_mentions(v, var) for v in expr)
    return False


# Built-in kernels (custom bodies): the positions of the tensor params they write.
_BUILTIN_OUTPUTS = {"paged_decode_gqa": {5}, "lightning_indexer_score": {3}, "topk_select": {1}}


def _written_params(plan: dict) -> dict[str, set[str]]:
    """kernel name -> names of the tensor params it writes (Store destinations; outputs of built-ins)."""
    res: dict[str, set[str]] = {}
    for k in plan["kernels"]:
        pid = {p["id"]: p["name"] for p in k["params"]}
        names = set()
        for op in k.get("ops", []):
            if op.get("kind") == "Store" and op["operands"] and op["operands"][0] in pid:
                names.add(pid[op["operands"][0]])
        src = str(k.get("attrs", {}).get("cpp_src", ""))
        first = src.lstrip().split("\n", 1)[0]
        if first.startswith("// ptowsp-builtin:"):
            builtin = first.split(":", 1)[1].strip()
            tparams = [p["name"] for p in k["params"]]
            for pos in _BUILTIN_OUTPUTS.get(builtin, ()):
                if pos < len(tparams):
                    names.add(tparams[pos])
        res[k["name"]] = names
    return res


def batch_tensors(plan: dict) -> tuple[set[int], set[int]]:
    """(tensors sliced by the outer axis, tensors read whole by every rank); see :func:`analyze`."""
    sliced, shared, _ = analyze(plan)
    return sliced, shared


def analyze(plan: dict) -> tuple[set[int], set[int], set[int]]:
    """(tensors sliced by the outer axis, tensors read whole by every rank, tensors written).

    A tensor is *sliced* when every access indexes its first dimension with
    the outer loop variable; *shared* when no access uses that variable.
    Anything else cannot be sharded and raises :class:`ShardError`: the
    variable in another index position, a shared tensor that is written, or a
    condition or inner axis that depends on the outer variable (a rank sees
    only local unit numbers).
    """
    written_by_kernel = _written_params(plan)
    sliced: set[int] = set()
    shared: set[int] = set()
    written: set[int] = set()
    for lp in outer_loops(plan):
        var = lp["var"]
        accesses: list[tuple[int, list]] = []

        def visit(n: dict) -> None:
            kind = n.get("kind")
            if kind == "task":
                outs = written_by_kernel.get(n["kernel"], set())
                for ta in n.get("tensor_args", []):
                    accesses.append((int(ta["tensor"]), ta.get("index", [])))
                    if ta["param"] in outs:
                        written.add(int(ta["tensor"]))
            elif kind == "slot_load":
                accesses.append((int(n["tensor_arg"]["tensor"]), n["tensor_arg"].get("index", [])))
            elif kind == "cond" and _mentions(n.get("pred"), var):
                raise ShardError(f"a condition depends on the outer variable {var!r}")
            elif kind in ("parallel_for", "for_each") and _mentions(n.get("axis"), var):
                raise ShardError(f"an inner axis depends on the outer variable {var!r}")

        _walk(lp["body"], visit)
        for tid, index in accesses:
            uses = [i for i, ix in enumerate(index) if _mentions(ix, var)]
            if uses == [0] and index[0].get("var") == var:
                sliced.add(tid)
            elif not uses:
                shared.add(tid)
            else:
                raise ShardError(f"tensor {tid} is indexed by an expression of the outer variable {var!r} "
                                 "other than its first index")
    both = sliced & shared
    if both:
        raise ShardError(f"tensors {sorted(both)} are both sliced by the outer axis and read whole")
    bad = shared & written
    if bad:
        raise ShardError(f"tensors {sorted(bad)} are written but not sliced by the outer axis: every rank would write them")
    return sliced, shared, written


def shard_plan(plan: dict, n_local: int) -> dict:
    """The plan a rank runs: outer static axes of size `n_local`, sliced tensors with first dimension `n_local`."""
    sliced, _ = batch_tensors(plan)
    p = copy.deepcopy(plan)
    for lp in outer_loops(p):
        if lp["axis"]["kind"] == "dense":
            lp["axis"]["size"] = int(n_local)
    for tid in sliced:
        p["tensors"][tid]["shape"][0] = int(n_local)
    p["name"] = f"{plan.get('name', 'workload')}_shard{n_local}"
    return p


# ---------------------------------------------------------------------------
# Partition
# ---------------------------------------------------------------------------


def partition(n: int, world: int, costs: Sequence[float] | None = None, method: str = "block") -> list[list[int]]:
    """Units 0..n-1 split over `world` ranks.

    ``block``: contiguous blocks, sizes differing by at most one (first ranks larger).
    ``balanced``: contiguous blocks whose cost sums are as even as a prefix split allows.
    ``lpt``: greedy longest-processing-time -- units by cost descending (ties: lower index first), each to the
    least-loaded rank (ties: lower rank); each rank's units in ascending order.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    if method == "block" or (method == "balanced" and costs is None):
        base, extra = divmod(n, world)
        out, lo = [], 0
        for r in range(world):
            hi = lo + base + (1 if r < extra else 0)
            out.append(list(range(lo, hi)))
            lo = hi
        return out
    if costs is None or len(costs) != n:
        raise ValueError(f"method {method!r} needs one cost per unit")
    c = [float(x) for x in costs]
    if method == "balanced":
        # the contiguous split whose largest share is smallest: bisection on that largest share, each probe a
        # greedy left-to-right fill, then the greedy split at the bound found
        def fill(cap: float) -> list[int]:
            cuts, acc = [], 0.0
            for i, x in enumerate(c):
                if acc + x > cap and acc > 0.0:
                    cuts.append(i)
                    acc = 0.0
                acc += x
            return cuts

        lo_cap, hi_cap = max(c, default=0.0), sum(c)
        for _ in range(60):
            mid = (lo_cap + hi_cap) / 2
            if len(fill(mid)) <= world - 1:
                hi_cap = mid
            else:
                lo_cap = mid
        cuts = fill(hi_cap)
        if n >= world:  # every rank gets a unit: extra cuts split segments, which raises no share
            taken = set(cuts)
            cuts = sorted(cuts + [i for i in range(1, n) if i not in taken][: world - 1 - len(cuts)])
        bounds = [0] + cuts + [n] * (world - len(cuts))
        return [list(range(bounds[r], bounds[r + 1])) for r in range(world)]
    if method == "lpt":
        order = sorted(range(n), key=lambda i: (-c[i], i))
        load = [0.0] * world
        out = [[] for _ in range(world)]
        for i in order:
            r = min(range(world), key=lambda k: (load[k], k))
            out[r].append(i)
            load[r] += c[i]
        return [sorted(u) for u in out]
    raise ValueError(f"unknown partition method {method!r}")


def _contiguous(units: list[int]) -> bool:
    return all(b == a + 1 for a, b in zip(units, units[1:]))


# ---------------------------------------------------------------------------
# Executable
# ---------------------------------------------------------------------------


def _dist():
    try:
        import torch.distributed as dist
    except ImportError:  # pragma: no cover
        return None
    return dist if dist.is_available() and dist.is_initialized() else None


_INDEX_CACHE: dict = {}  # (device, units) -> index tensor on that device (made once, not per run)


def _index(units: list[int], device: Any) -> Any:
    import torch

    key = (str(device), tuple(units))
    t = _INDEX_CACHE.get(key)
    if t is None:
        if len(_INDEX_CACHE) > 256:
            _INDEX_CACHE.clear()
        t = _INDEX_CACHE[key] = torch.as_tensor(units, device=device, dtype=torch.long)
    return t


def _take(a: Any, units: list[int]) -> Any:
    if _contiguous(units):
        lo = units[0] if units else 0
        return a[lo:lo + len(units)]
    if hasattr(a, "index_select"):
        return a.index_select(0, _index(units, a.device))
    import numpy as np

    return np.ascontiguousarray(a[np.asarray(units, dtype=np.int64)])


def _put(a: Any, units: list[int], local: Any) -> None:
    if _contiguous(units):
        return  # the rank wrote through a view
    if hasattr(a, "index_copy_"):
        a.index_copy_(0, _index(units, a.device), local)
        return
    import numpy as np

    a[np.asarray(units, dtype=np.int64)] = local


class ShardedExecutable:
    """One rank's share of a plan whose outermost ``P()`` axis is split over the ranks.

    ``arrays`` passed to :meth:`run_with_symbols` are the *global* tensors (host numpy or CUDA torch tensors);
    the rank runs its units, writes its slice of every output in place, and -- for the tensor ids in
    ``gather`` (replicated layouts) -- gathers the other ranks' slices so that every rank ends up with the whole
    tensor.  Without ``gather`` no collective runs.
    """

    def __init__(self, plan: dict, rank: int | None = None, world: int | None = None, device: int | None = None,
                 method: str = "block", costs: Sequence[float] | None = None, gather: Sequence[int] = (),
                 group: Any = None, executable_factory: Callable[[dict, int], Any] | None = None):
        dist = _dist()
        self.rank = rank if rank is not None else (dist.get_rank(group) if dist else int(os.environ.get("RANK", 0)))
        self.world = world if world is not None else (
            dist.get_world_size(group) if dist else int(os.environ.get("WORLD_SIZE", 1)))
        if not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside world {self.world}")
        self.device = device if device is not None else int(os.environ.get("LOCAL_RANK", self.rank))
        self.plan = plan
        self.loops = outer_loops(plan)
        self.var_names = [lp["var"] for lp in self.loops]
        self.n_static = _outer_size(self.loops)
        self.sliced, self.shared, self.written = analyze(plan)
        self.method, self.costs = method, costs
        self.gather = [int(t) for t in gather]
        for t in self.gather:
            if t not in self.sliced:
                raise ShardError(f"tensor {t} is not sliced by the outer axis: nothing to gather")
        self.group = group
        if executable_factory is None:
            from .runtime import CudaExecutable

            executable_factory = lambda p, dev: CudaExecutable(p, device=dev)  # noqa: E731
        self._factory = executable_factory
        self._exes: dict[int, Any] = {}
        self.units: list[list[int]] | None = None
        self.last_gather_ms = 0.0
        if self.n_static is not None:
            self.units = partition(self.n_static, self.world, costs, method)

    def local_units(self, n: int | None = None) -> list[int]:
        if self.n_static is None:
            if n is None:
                raise ShardError("the outer axis is DenseDyn: give its size in axis_sizes")
            if getattr(self, "_units_n", None) != n:  # the split depends only on n (and the fixed costs)
                self.units = partition(n, self.world, self.costs[:n] if self.costs is not None else None, self.method)
                self._units_n = n
        return self.units[self.rank]

    def executable(self, n_local: int) -> Any:
        if n_local not in self._exes:
            self._exes[n_local] = self._factory(shard_plan(self.plan, n_local), self.device)
        return self._exes[n_local]

    def run_with_symbols(self, arrays: Sequence[Any], axis_sizes: dict | None = None, symbols_u64: dict | None = None,
                         symbols_ptr: dict | None = None) -> int:
        axis_sizes = dict(axis_sizes or {})
        n = None
        if self.n_static is None:
            sizes = {axis_sizes.get(v) for v in self.var_names}
            if len(sizes) != 1 or None in sizes:
                raise ShardError(f"DenseDyn outer axis: axis_sizes must give {self.var_names}")
            n = int(sizes.pop())
        units = self.local_units(n)
        local = [(_take(a, units) if i in self.sliced else a) for i, a in enumerate(arrays)]
        for v in self.var_names:
            if v in axis_sizes:
                axis_sizes[v] = len(units)
        cycles = 0
        if units:
            cycles = self.executable(len(units)).run_with_symbols(local, axis_sizes, symbols_u64 or {}, symbols_ptr or {})
            for i in self.sliced & self.written:
                _put(arrays[i], units, local[i])
        self.last_gather_ms = 0.0
        if self.gather and self.world > 1:
            t0 = time.perf_counter()
            for t in self.gather:
                allgather_units(arrays[t], self.units, self.rank, self.group)
            self.last_gather_ms = (time.perf_counter() - t0) * 1e3
        return cycles

    def run(self, arrays: Sequence[Any], axis_sizes: dict | None = None) -> int:
        return self.run_with_symbols(arrays, axis_sizes)


def allgather_units(a: Any, units: list[list[int]], rank: int, group: Any = None) -> None:
    """Every rank's rows `units[r]` of `a` (first dimension) end up in every rank's `a`.

    Rows are padded to the largest share so that one ``all_gather`` moves them.  With an NCCL group the exchange
    runs on CUDA tensors (host arrays are staged through the current device); with gloo, on host tensors.
    """
    import numpy as np
    import torch
    import torch.distributed as dist

    world = len(units)
    t = torch.from_numpy(a) if isinstance(a, np.ndarray) else a
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    maxn = max(len(u) for u in units)
    row = tuple(t.shape[1:])
    mine = units[rank]
    buf = torch.zeros((maxn,) + row, dtype=t.dtype, device=dev)
    if mine:
        src = t.index_select(0, torch.as_tensor(mine, dtype=torch.long, device=t.device))
        buf[: len(mine)] = src.to(dev)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    for r, u in enumerate(units):
        if r == rank or not u:
            continue
        idx = torch.as_tensor(u, dtype=torch.long, device=t.device)
        t.index_copy_(0, idx, parts[r][: len(u)].to(t.device))
