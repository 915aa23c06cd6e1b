"""The allocation-free paged-decode entry point (-m gpu).

`ptowsp_cuda_paged_decode_noalloc` is for callers that must not let a library
allocate device memory during a call -- serving engines whose memory is fully
reserved up front by their own KV-cache pool, or hosts that cannot take the
synchronisation cudaMalloc/cudaFree can cause.  It keeps its scratch in one
fixed array of device memory owned by the library.

This test calls it through the C ABI twice in a row (the second call with other
lengths, so stale scratch from the first call would show) and checks each
result against the CPU oracle's decode task (the decode tests' tolerance) and
bit for bit against the regular entry point (`ptowsp_cuda_main` on the decode
plan, same kernels).  It also checks that calls after the first take no device
memory, a later one with another GQA group included, and that a workload too
big for the fixed array is refused.  The file name makes pytest collect it last.
"""

import ctypes as C

import numpy as np
import pytest
from cpu_sim import CpuSim

from tolerance import RTOL_F16_MMA, assert_rel, rms

from pto_wsp_b200 import workloads
from pto_wsp_b200.runtime import CudaExecutable, load_library

pytestmark = pytest.mark.gpu


def check(got, ref):
    ref = np.asarray(ref, np.float64)
    assert_rel(got, ref, RTOL_F16_MMA, 5e-2 * rms(ref))


def oracle(plan, arrays, R):
    ref = [a.copy() for a in arrays]
    CpuSim(plan).run(ref, axis_sizes={"b": R})
    return ref[5]


def noalloc_fn():
    lib = load_library()
    f = lib.ptowsp_cuda_paged_decode_noalloc
    f.argtypes = [C.c_void_p] * 6 + [C.c_int] * 6 + [C.c_int64, C.c_void_p]
    f.restype = C.c_int
    need = lib.ptowsp_cuda_noalloc_scratch_bytes
    need.argtypes = [C.c_int] * 5
    need.restype = C.c_size_t
    return lib, f, need


def to_device(torch, arrays):
    q, kc, vc, pt, kl, out = arrays
    dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (q, kc, vc, pt, kl.reshape(-1), out)]
    dev[5].fill_(float("nan"))
    torch.cuda.synchronize()
    return dev


def call_noalloc(f, torch, dev, R, KVH=8, G=4, D=128, page=16):
    return f(*[t.data_ptr() for t in dev], R, KVH, G, D, page, dev[3].shape[1], dev[1].shape[0],
             torch.cuda.current_stream().cuda_stream)


def run_regular(plan, arrays, R):
    got = [a.copy() for a in arrays]
    CudaExecutable(plan).run_with_symbols(got, {"b": R}, {}, {})
    return got[5]


def test_noalloc_matches_oracle_and_regular_entry_point_twice(require_cuda):
    torch = pytest.importorskip("torch")
    lib, f, need = noalloc_fn()
    rng = np.random.default_rng(7)
    R = 12
    plan1, a1 = workloads.decode_inputs(rng, R, lo=1, hi=3000, max_pages=200)
    plan2, a2 = workloads.decode_inputs(rng, R, lengths=[0, 1, 17, 513, 2000, 3199, 5, 64, 1024, 700, 16, 3000],
                                        max_pages=200)
    assert need(R, 8, 4, 200, 16) <= need(0, 0, 0, 0, 0)

    d1 = to_device(torch, a1)
    rc = call_noalloc(f, torch, d1, R)
    assert rc == 0, lib.ptowsp_cuda_last_error()
    out1 = d1[5].cpu().numpy()
    check(out1, oracle(plan1, a1, R))
    np.testing.assert_array_equal(out1, run_regular(plan1, a1, R))

    d2 = to_device(torch, a2)  # inputs of the second call are allocated by the test, before measuring
    free_before = torch.cuda.mem_get_info()[0]
    rc = call_noalloc(f, torch, d2, R)
    free_after = torch.cuda.mem_get_info()[0]
    assert rc == 0, lib.ptowsp_cuda_last_error()
    assert free_after == free_before  # the call itself took no device memory
    out2 = d2[5].cpu().numpy()
    assert not np.isnan(out2.astype(np.float32)).any()
    check(out2, oracle(plan2, a2, R))
    np.testing.assert_array_equal(out2, run_regular(plan2, a2, R))


def test_noalloc_other_group_takes_no_memory(require_cuda):
    torch = pytest.importorskip("torch")
    lib, f, need = noalloc_fn()
    rng = np.random.default_rng(9)
    # a first call with GQA group 4 (the first on this device when the test runs alone: it sets the device up)
    _, a4 = workloads.decode_inputs(rng, 3, lengths=[10, 600, 2000])
    d4 = to_device(torch, a4)
    assert call_noalloc(f, torch, d4, 3) == 0, lib.ptowsp_cuda_last_error()
    # then group 2 and group 8, which no earlier call launched: no device memory either
    for KVH, G in ((4, 2), (2, 8)):
        R = 5
        plan, arrays = workloads.decode_inputs(rng, R, kv_heads=KVH, group=G, lengths=[1, 700, 1600, 33, 4000])
        d = to_device(torch, arrays)
        free_before = torch.cuda.mem_get_info()[0]
        rc = call_noalloc(f, torch, d, R, KVH=KVH, G=G)
        free_after = torch.cuda.mem_get_info()[0]
        assert rc == 0, lib.ptowsp_cuda_last_error()
        assert free_after == free_before, (G, free_before - free_after)
        check(d[5].cpu().numpy(), oracle(plan, arrays, R))


def test_noalloc_rejects_work_beyond_the_fixed_array(require_cuda):
    torch = pytest.importorskip("torch")
    lib, f, need = noalloc_fn()
    cap = need(0, 0, 0, 0, 0)
    R, KVH, G, maxp = 512, 8, 8, 4096  # far more partials than the array holds
    assert need(R, KVH, G, maxp, 16) > cap
    x = torch.zeros(16, dtype=torch.float16, device="cuda")
    rc = f(*([x.data_ptr()] * 6), R, KVH, G, 128, 16, maxp, 1, None)
    assert rc == 6
    assert b"24 MiB" in lib.ptowsp_cuda_last_error()
