"""Sharding the outermost P(batch) axis (pto_wsp_b200.shard), on the CPU.

* partitions cover every unit exactly once (block, cost-balanced blocks, LPT);
* the loop-nest analysis finds the sliced / shared / written tensors of the
  five BASELINE plans and refuses nests that cannot be split;
* a rank's plan (outer size and sliced shapes rewritten) computes, on the
  oracle, exactly the rank's slice of the whole-batch result;
* two gloo ranks (separate processes, 127.0.0.1) run their shares and gather
  the replicated outputs (contiguous blocks and a non-contiguous LPT split).
"""

import copy
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
from cpu_sim import CpuSim

from pto_wsp_b200 import shard, workloads

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("n,world", [(10, 3), (3, 4), (0, 2), (64, 8), (1, 1)])
def test_block_partition_covers_units(n, world):
    parts = shard.partition(n, world)
    assert [u for p in parts for u in p] == list(range(n))
    sizes = [len(p) for p in parts]
    assert max(sizes) - min(sizes) <= 1


def test_balanced_and_lpt_partitions():
    rng = np.random.default_rng(0)
    costs = rng.integers(512, 8193, 64).tolist()
    for method in ("balanced", "lpt"):
        parts = shard.partition(64, 8, costs, method)
        assert sorted(u for p in parts for u in p) == list(range(64))
        loads = [sum(costs[u] for u in p) for p in parts]
        assert max(loads) <= sum(costs) / 8 + max(costs)  # within one unit of the even share
    lpt = shard.partition(6, 2, [5, 1, 4, 2, 3, 3], "lpt")
    assert lpt == [[0, 1, 5], [2, 3, 4]]
    bal = shard.partition(4, 2, [1, 1, 1, 9], "balanced")
    assert bal == [[0, 1, 2], [3]]


def test_balanced_partition_minimises_the_largest_share():
    import itertools

    rng = np.random.default_rng(5)
    for _ in range(30):
        n = int(rng.integers(3, 11))
        world = int(rng.integers(2, min(n, 4) + 1))
        costs = rng.integers(1, 100, n).tolist()
        parts = shard.partition(n, world, costs, "balanced")
        assert [u for p in parts for u in p] == list(range(n))  # contiguous, in order
        assert all(parts)  # every rank has a unit (n >= world here)
        got = max(sum(costs[u] for u in p) for p in parts)
        best = min(max(sum(costs[a:b]) for a, b in zip((0,) + cut, cut + (n,)))
                   for cut in itertools.combinations(range(1, n), world - 1))
        assert got == best


def test_analysis_of_the_config_plans():
    assert shard.analyze(workloads.rmsnorm_plan(4, 8)) == ({0, 1}, set(), {1})
    assert shard.analyze(workloads.softmax_plan(4, 8)) == ({0, 1}, set(), {1})
    assert shard.analyze(workloads.bgemm_plan(2, 256, 256, 128)) == ({0, 1, 2}, set(), {2})
    assert shard.analyze(workloads.decode_plan(5, 8, 4, 128, 100, 20)) == ({0, 3, 4, 5}, {1, 2}, {5})
    assert shard.analyze(workloads.indexer_plan(4, 8, 64, 128, 256, 16)) == ({0, 1, 2, 3, 4}, set(), {3, 4})


def test_nests_that_cannot_be_split_are_refused():
    p = workloads.rmsnorm_plan(4, 8)
    bad = copy.deepcopy(p)
    bad["body"]["body"]["body"]["tensor_args"][1]["index"] = [{"var": "h"}, {"var": "b"}]  # out[t][b]
    with pytest.raises(shard.ShardError):
        shard.analyze(bad)
    shared_out = copy.deepcopy(p)
    shared_out["body"]["body"]["body"]["tensor_args"][1]["index"] = [{"const": 0}, {"var": "h"}]  # out[0][t]
    with pytest.raises(shard.ShardError, match="written but not sliced"):
        shard.analyze(shared_out)
    seq = copy.deepcopy(p)
    seq["body"] = {"kind": "sequential", "children": [p["body"], workloads.rmsnorm_plan(5, 8)["body"]]}
    with pytest.raises(shard.ShardError, match="different sizes"):
        shard.ShardedExecutable(seq, rank=0, world=2, executable_factory=lambda pl, d: None)


def test_rank_plans_compute_their_slice_on_the_oracle():
    rng = np.random.default_rng(1)
    plan = workloads.rmsnorm_plan(5, 4)
    x = rng.standard_normal((5, 4, 16, 128)).astype(np.float32)
    whole = np.zeros_like(x)
    CpuSim(plan).run([x, whole])
    for units in shard.partition(5, 2):
        lo, hi = units[0], units[-1] + 1
        sp = shard.shard_plan(plan, len(units))
        assert sp["tensors"][0]["shape"] == [len(units), 4, 16, 128]
        part = np.zeros_like(x[lo:hi])
        CpuSim(sp).run([np.ascontiguousarray(x[lo:hi]), part])
        np.testing.assert_array_equal(part, whole[lo:hi])


def test_decode_plan_shards_requests_by_kv_length():
    rng = np.random.default_rng(2)
    plan, arrays = workloads.decode_inputs(rng, 6, lengths=[100, 900, 40, 700, 300, 500])
    lens = arrays[4].reshape(-1).tolist()
    whole = [a.copy() for a in arrays]
    CpuSim(plan).run(whole, axis_sizes={"b": 6})
    got = [a.copy() for a in arrays]
    got[5][...] = 0
    for rank in range(2):
        class OracleChecker:  # runs the rank's plan on the oracle so its result can be compared with the whole run
            def __init__(self, p, d):
                self.p = p

            def run_with_symbols(self, arrs, ax, su, sp):
                return CpuSim(self.p).run(arrs, axis_sizes=ax)

        ex = shard.ShardedExecutable(plan, rank=rank, world=2, method="lpt", costs=lens,
                                     executable_factory=OracleChecker)
        ex.run_with_symbols(got, {"b": 6})
        assert ex.units == [[0, 1, 4], [2, 3, 5]]  # LPT over 900, 700, 500, 300, 100, 40
    np.testing.assert_array_equal(got[5], whole[5])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_shard_and_gather():
    port = _free_port()
    procs = []
    for rank in range(2):
        env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                   LOCAL_RANK=str(rank))
        procs.append(subprocess.Popen([sys.executable, str(ROOT / "tests" / "_shard_worker.py")], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=180)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append(out)
    for rank, (p, out) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, out
        assert f"rank {rank} ok" in out
