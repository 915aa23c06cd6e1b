"""One rank of the 2-GPU NCCL test in tests/test_gpu_shard.py (not collected)."""

import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from pto_wsp_b200 import shard, workloads  # noqa: E402
from pto_wsp_b200.runtime import CudaExecutable  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    rank = dist.get_rank()
    g = torch.Generator(device=dev)
    g.manual_seed(11)  # the same global input on both ranks
    x = torch.randn((5, 32, 32, 256), device=dev, generator=g) * 4
    plan = workloads.softmax_plan(5, 32)
    ex = shard.ShardedExecutable(plan, gather=[1])
    y = torch.full_like(x, float("nan"))
    ex.run_with_symbols([x, y], {})
    whole = torch.empty_like(x)
    CudaExecutable(plan, device=local).run_with_symbols([x, whole], {}, {}, {})
    assert torch.equal(y, whole), "gathered output differs from the single-rank run"
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()
    print(f"rank {rank} ok (gather {ex.last_gather_ms:.3f} ms)", flush=True)


if __name__ == "__main__":
    main()
