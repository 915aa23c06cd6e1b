"""Sharded runs on the GPU (-m gpu).

Single GPU: the ranks of a 2-way split run one after the other on device 0
through the real CUDA executable; together they must reproduce the unsharded
run bit for bit (every unit is computed by the same kernel either way).
Two GPUs (skipped with fewer): two NCCL ranks, one per GPU, run their shares
of device-resident tensors and all-gather the replicated output.
"""

import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from pto_wsp_b200 import shard, workloads
from pto_wsp_b200.runtime import CudaExecutable

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def test_decode_lpt_shares_reproduce_the_whole_run(require_cuda):
    rng = np.random.default_rng(3)
    lengths = [4000, 17, 900, 2500, 0, 1536, 3000, 77]
    plan, arrays = workloads.decode_inputs(rng, len(lengths), lengths=lengths)
    whole = [a.copy() for a in arrays]
    CudaExecutable(plan).run_with_symbols(whole, {"b": len(lengths)}, {}, {})
    got = [a.copy() for a in arrays]
    got[5][...] = np.float16(np.nan)
    for rank in range(2):
        ex = shard.ShardedExecutable(plan, rank=rank, world=2, device=0, method="lpt", costs=lengths)
        ex.run_with_symbols(got, {"b": len(lengths)})
    assert sorted(ex.units[0] + ex.units[1]) == list(range(len(lengths)))
    assert not all(b == a + 1 for a, b in zip(ex.units[0], ex.units[0][1:]))  # a non-contiguous share
    np.testing.assert_array_equal(got[5], whole[5])


def test_rmsnorm_block_shares_on_device_tensors(require_cuda):
    torch = pytest.importorskip("torch")
    x = torch.randn((6, 64, 16, 128), device="cuda")
    whole = torch.empty_like(x)
    plan = workloads.rmsnorm_plan(6, 64)
    CudaExecutable(plan).run_with_symbols([x, whole], {}, {}, {})
    y = torch.full_like(x, float("nan"))
    for rank in range(3):
        shard.ShardedExecutable(plan, rank=rank, world=3, device=0).run_with_symbols([x, y], {})
    assert torch.equal(y, whole)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_nccl_ranks_gather_the_replicated_output(require_cuda):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = _free_port()
    procs = []
    for rank in range(2):
        env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                   LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, str(ROOT / "tests" / "_shard_nccl_worker.py")], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=300)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append(out)
    for rank, (p, out) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, out
        assert f"rank {rank} ok" in out
