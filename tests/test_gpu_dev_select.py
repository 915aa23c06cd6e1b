"""`P.when` tiers over a slot loaded from a tensor, decided on the GPU (-m gpu).

The walk places one task per iteration and a small kernel picks each task's scalars from the tensor element before
the batch runs, so a tensor that changes between runs changes the chosen tier without a new walk or any host read of
the data.  Checked against the oracle, which evaluates the conds on the host like the reference CPU-sim."""

import numpy as np
import pytest
from _dev_select import expected_scale, tiered_scale_plan
from cpu_sim import CpuSim

from pto_wsp_b200.runtime import CudaExecutable

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("src_dtype,slot_type", [("i32", "i64"), ("u32", "u64"), ("i64", "i64"), ("f32", "i64")])
def test_device_selected_tiers_follow_the_tensor(src_dtype, slot_type, require_cuda):
    torch = pytest.importorskip("torch")
    B, T = 6, 40
    plan = tiered_scale_plan(B, T, src_dtype=src_dtype, slot_type=slot_type)
    ex = CudaExecutable(plan)
    assert ex.describe()["cacheable"]
    rng = np.random.default_rng(len(src_dtype) + len(slot_type))
    x = rng.standard_normal((B, T, 8, 64)).astype(np.float32)
    npdt = {"i32": np.int32, "u32": np.uint32, "i64": np.int64, "f32": np.float32}[src_dtype]
    xd = torch.from_numpy(x).cuda()
    out = torch.full_like(xd, float("nan"))
    seld = None
    for run in range(3):
        lo = 0 if src_dtype == "u32" else -30
        sel = rng.integers(lo, 250, (B, T, 1, 1)).astype(npdt)
        if seld is None:
            seld = torch.from_numpy(sel).cuda()
        else:
            seld.copy_(torch.from_numpy(sel))  # same device buffer, new values: the cached task table is replayed
        want = np.full_like(x, np.nan)
        cyc = CpuSim(plan).run([sel, x, want])
        assert ex.run_with_symbols([seld, xd, out], {}, {}, {}) == cyc
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), want)
        assert ex.timing()["slot_syncs"] == 0  # no host read of the tensor
        if src_dtype in ("i32", "i64"):
            scales = np.vectorize(expected_scale)(sel.astype(np.int64)).astype(np.float32)
            np.testing.assert_array_equal(want, x * scales)


def test_device_selected_tiers_with_host_arrays(require_cuda):
    B, T = 4, 9
    plan = tiered_scale_plan(B, T)
    rng = np.random.default_rng(3)
    sel = rng.integers(-30, 250, (B, T, 1, 1)).astype(np.int32)
    x = rng.standard_normal((B, T, 8, 64)).astype(np.float32)
    want = np.zeros_like(x)
    cyc = CpuSim(plan).run([sel, x, want])
    got = np.full_like(x, np.nan)
    assert CudaExecutable(plan).run_with_symbols([sel, x, got], {}, {}, {}) == cyc
    np.testing.assert_array_equal(got, want)
