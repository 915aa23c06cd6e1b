"""The five BASELINE configs split over 2, 4 and 8 ranks (host only).

``bench.py --gpus N`` runs each rank's ``ShardedExecutable`` share of the one global config.  Here every rank of
every world size the scaling bench uses takes its share on the host: the shares cover the outer ``P(batch)`` axis
exactly once, no rank is left without work, config 4's KV-length-balanced shares stay close to the mean, and each
rank's plan walks through the native runtime (``dry_run``: walk, waves and staging, no device) with the rank's task
count, so that the tasks of all ranks add up to those of the unsharded run.  Inputs are zero-filled numpy arrays of
the global shapes (config 4 with its real page table and lengths, which the walk reads).
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from pto_wsp_b200 import runtime  # noqa: E402
from pto_wsp_b200.shard import ShardedExecutable  # noqa: E402

_DT = {"f32": np.float32, "f16": np.float16, "i32": np.int32}


def _case(name: str):
    return bench.CASES[name](argparse.Namespace(batch=None, cols=None, partition=None))


def _arrays(case, plan: dict) -> list[np.ndarray]:
    arrs = [np.zeros(t["shape"], _DT[t["dtype"]]) for t in plan["tensors"]]
    if case.name == "decode":  # page table and KV lengths: the walk reads them
        arrs[3][...] = case.pt
        arrs[4][:, 0] = case.lens
    return arrs


def _dry(plan: dict, _device: int):
    ex = runtime.CudaExecutable(plan)
    ex.set_option("dry_run", 1)
    return ex


@pytest.fixture(scope="module")
def unsharded_tasks() -> dict[str, int]:
    out = {}
    for name in bench.ORDER:
        case = _case(name)
        plan = case.plan()
        ex = _dry(plan, 0)
        ex.run_with_symbols(_arrays(case, plan), case.axis(case.n_units), {}, {})
        out[name] = int(ex.timing()["tasks"])
    return out


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("name", bench.ORDER)
def test_every_rank_plans_its_share(name, world, unsharded_tasks):
    case = _case(name)
    plan = case.plan()
    arrays = _arrays(case, plan)
    shares, tasks = [], 0
    for rank in range(world):
        sh = ShardedExecutable(plan, rank=rank, world=world, device=0, method=case.method, costs=case.costs(),
                               executable_factory=_dry)
        units = sh.local_units(case.n_units)
        assert units, f"{name}: rank {rank} of {world} has no units"
        shares.append(units)
        sh.run_with_symbols(arrays, case.axis(case.n_units))
        tasks += int(sh.executable(len(units)).timing()["tasks"])
    flat = [u for s in shares for u in s]
    assert sorted(flat) == list(range(case.n_units))
    if case.method in ("block", "balanced"):  # contiguous shares: each rank works on views of the global tensors
        assert all(s == list(range(s[0], s[0] + len(s))) for s in shares)
    assert tasks == unsharded_tasks[name]
    if name == "decode":
        loads = [float(case.lens[s].sum()) for s in shares]
        assert max(loads) / (sum(loads) / world) < 1.12
