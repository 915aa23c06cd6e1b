"""Paged GQA decode vs the oracle / fp64 (-m gpu).

Tolerance: f16 output of an f32 softmax over f16 K/V, against the oracle's fp64 task: plain relative error
<= 2e-3 (the north_star's bar for f16 contractions) on every element with |O64| >= 5e-2 rms(O64); smaller
elements within 2e-3 x that floor.  At full size every request is recomputed in fp64 on the GPU.
"""

import numpy as np
import pytest
from cpu_sim import CpuSim

from tolerance import RTOL_F16_MMA, assert_rel, rms

from pto_wsp_b200 import workloads
from pto_wsp_b200.runtime import CudaExecutable

pytestmark = pytest.mark.gpu
FLOOR = 5e-2


def check(got, ref):
    ref = np.asarray(ref, np.float64)
    return assert_rel(got, ref, RTOL_F16_MMA, FLOOR * rms(ref))


@pytest.mark.parametrize("lengths", [[0, 1, 16, 17, 512, 513, 1024, 1500], [700, 33, 2049]])
def test_decode_edge_lengths_vs_oracle(lengths, require_cuda):
    rng = np.random.default_rng(0)
    plan, arrays = workloads.decode_inputs(rng, len(lengths), lengths=lengths)
    ref = [a.copy() for a in arrays]
    cyc = CpuSim(plan).run(ref, axis_sizes={"b": len(lengths)})
    ex = CudaExecutable(plan)
    assert ex.describe()["kernels"][0]["impl"] == "paged_decode_gqa"
    got = [a.copy() for a in arrays]
    got[5][...] = np.float16(np.nan)
    assert ex.run_with_symbols(got, {"b": len(lengths)}, {}, {}) == cyc
    check(got[5], ref[5])
    assert not np.isnan(got[5].astype(np.float32)).any()
    # L = 0 -> zeros, as the oracle
    for r, L in enumerate(lengths):
        if L == 0:
            assert not got[5][r].any()
    # device-resident output pre-filled with NaN: every element is written, zeros for L = 0 included
    torch = pytest.importorskip("torch")
    dev = [torch.from_numpy(a.copy()).cuda() for a in arrays]
    dev[5].fill_(float("nan"))
    ex.run_with_symbols(dev, {"b": len(lengths)}, {}, {})
    check(dev[5].cpu().numpy(), ref[5])


@pytest.mark.parametrize("chunk", [512, 768, 1024, 1536, 1000])
def test_decode_split_kv_chunk_lengths_vs_oracle(chunk, require_cuda):
    """Every split-KV chunk length the launch may choose (the `decode_chunk` option forces one; 1000 is taken as
    992, a multiple of 16), over lengths on either side of each chunk boundary: the chunk partials merge to the
    oracle's result."""
    lengths = [0, 1, 511, 512, 513, 767, 768, 769, 992, 993, 1535, 1536, 1537, 3000, 4097]
    rng = np.random.default_rng(chunk)
    plan, arrays = workloads.decode_inputs(rng, len(lengths), lengths=lengths)
    ref = [a.copy() for a in arrays]
    CpuSim(plan).run(ref, axis_sizes={"b": len(lengths)})
    ex = CudaExecutable(plan)
    ex.set_option("decode_chunk", chunk)
    got = [a.copy() for a in arrays]
    got[5][...] = np.float16(np.nan)
    ex.run_with_symbols(got, {"b": len(lengths)}, {}, {})
    check(got[5], ref[5])
    assert not got[5][0].any()


def test_decode_dense_dyn_axis_runs_fewer_requests(require_cuda):
    rng = np.random.default_rng(1)
    plan, arrays = workloads.decode_inputs(rng, 5, lengths=[100, 200, 300, 400, 500])
    got = [a.copy() for a in arrays]
    ex = CudaExecutable(plan)
    ex.run_with_symbols(got, {"b": 3}, {}, {})  # only requests 0..2 (DenseDyn bound at run time)
    ref = [a.copy() for a in arrays]
    CpuSim(plan).run(ref, axis_sizes={"b": 3})
    check(got[5], ref[5])
    assert not got[5][3:].any()


def test_decode_dense_dyn_axis_of_size_zero(require_cuda):
    # no request at all: no task, no launch, the output comes back as it went in (the oracle's 0 cycles)
    rng = np.random.default_rng(2)
    plan, arrays = workloads.decode_inputs(rng, 3, lengths=[10, 20, 30])
    got = [a.copy() for a in arrays]
    got[5][...] = np.float16(1.5)
    ex = CudaExecutable(plan)
    assert ex.run_with_symbols(got, {"b": 0}, {}, {}) == CpuSim(plan).run([a.copy() for a in arrays],
                                                                          axis_sizes={"b": 0}) == 0
    assert ex.timing()["launches"] == 0 and ex.timing()["tasks"] == 0
    assert np.all(got[5] == np.float16(1.5))
    ex.run_with_symbols(got, {"b": 2}, {}, {})  # the same executable then runs a non-empty share
    ref = [a.copy() for a in arrays]
    ref[5][...] = np.float16(1.5)
    CpuSim(plan).run(ref, axis_sizes={"b": 2})
    check(got[5][:2], ref[5][:2])
    assert np.all(got[5][2] == np.float16(1.5))


def test_decode_config4_full_size(require_cuda):
    import math

    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(4)
    R = 64
    plan, arrays = workloads.decode_inputs(rng, R)  # KV lengths U{512..8192}, 8 kv heads, GQA 4, d=128
    dev = [torch.from_numpy(a).cuda() for a in arrays]
    dev[5].fill_(float("nan"))
    ex = CudaExecutable(plan)
    ex.run_with_symbols(dev, {"b": R}, {}, {})
    out = dev[5].cpu().numpy()
    # the oracle's own task (numpy, fp64) on two requests ...
    for r in (0, 63):
        one = [a.copy() for a in arrays]
        CpuSim(plan).run(one, axis_sizes={"b": r + 1})
        check(out[r], one[5][r])
    # ... and every request recomputed in fp64 on the GPU through the same page walk
    q, kc, vc, pt, kl = dev[:5]
    lens = arrays[4].reshape(-1)
    for r in range(R):
        L = int(lens[r])
        pages = pt[r, : (L + 15) // 16].long()
        k = kc[pages].reshape(-1, 8, 128)[:L].double()
        v = vc[pages].reshape(-1, 8, 128)[:L].double()
        s = torch.einsum("hgd,thd->hgt", q[r].double(), k) / math.sqrt(128)
        ref = torch.einsum("hgt,thd->hgd", torch.softmax(s, -1), v).cpu().numpy()
        check(out[r], ref)


@pytest.mark.parametrize("group", [1, 2, 8])
def test_decode_gqa_groups_vs_oracle(group, require_cuda):
    rng = np.random.default_rng(10 + group)
    lengths = [1, 513, 1100, 2049, 16]
    plan, arrays = workloads.decode_inputs(rng, len(lengths), kv_heads=4, group=group, lengths=lengths)
    ref = [a.copy() for a in arrays]
    cyc = CpuSim(plan).run(ref, axis_sizes={"b": len(lengths)})
    ex = CudaExecutable(plan)
    for _ in range(2):  # the second run reuses the per-task arrival counters of the first
        got = [a.copy() for a in arrays]
        got[5][...] = np.float16(np.nan)
        assert ex.run_with_symbols(got, {"b": len(lengths)}, {}, {}) == cyc
        check(got[5], ref[5])
