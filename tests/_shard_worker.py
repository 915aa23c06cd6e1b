"""One rank of the 2-process gloo test of pto_wsp_b200.shard (run by tests/test_shard.py, not collected).

Each rank holds the same seeded global arrays, runs its share of the units
through ShardedExecutable with a small numpy stand-in for the per-rank CUDA
executable (this is a host-logic test: partition, plan rewrite, slicing,
scatter, gather), gathers the replicated outputs, and checks them against
the same computation over the whole batch.
"""

import os
import sys

import numpy as np
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from pto_wsp_b200 import shard, workloads  # noqa: E402


class RowsStandIn:
    """Numpy stand-in of the per-rank executable for the RMSNorm and top-k plans."""

    def __init__(self, plan, device):
        self.plan = plan

    def run_with_symbols(self, arrays, axis_sizes, su, sp):
        for t, a in zip(self.plan["tensors"], arrays):
            assert list(a.shape) == t["shape"], (a.shape, t["shape"])
        if self.plan["kernels"][0]["name"] == "rmsnorm_tile":
            x, y = arrays
            y[...] = x / np.sqrt((x * x).mean(-1, keepdims=True))
        else:
            s, out = arrays
            k = out.shape[-1]
            for r in range(s.shape[0]):
                out[r, 0] = np.lexsort((np.arange(s.shape[-1]), -s[r, 0].astype(np.float64)))[:k]
        return 1


def main():
    dist.init_process_group("gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    rng = np.random.default_rng(0)
    # RMSNorm, contiguous blocks (5 batch elements over 2 ranks: 3 + 2), output replicated
    x = rng.standard_normal((5, 3, 16, 128)).astype(np.float32)
    y = np.zeros_like(x)
    ex = shard.ShardedExecutable(workloads.rmsnorm_plan(5, 3), gather=[1], executable_factory=RowsStandIn)
    assert ex.local_units() == ([0, 1, 2] if rank == 0 else [3, 4])
    ex.run_with_symbols([x, y], {})
    np.testing.assert_allclose(y, x / np.sqrt((x * x).mean(-1, keepdims=True)), rtol=1e-6)
    # top-k rows, longest-processing-time partition by a per-row cost: non-contiguous shares
    s = rng.standard_normal((7, 1, 300)).astype(np.float32)
    idx = np.full((7, 1, 9), -1, np.int32)
    costs = [5, 1, 4, 2, 3, 3, 9]
    ex2 = shard.ShardedExecutable(workloads.topk_plan(7, 300, 9), method="lpt", costs=costs, gather=[1],
                                  executable_factory=RowsStandIn)
    assert sorted(ex2.units[0] + ex2.units[1]) == list(range(7))
    ex2.run_with_symbols([s, idx], {})
    for r in range(7):
        assert idx[r, 0].tolist() == np.lexsort((np.arange(300), -s[r, 0].astype(np.float64)))[:9].tolist()
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank} ok", flush=True)


if __name__ == "__main__":
    main()
