"""The allocation-free paged-decode entry point (-m gpu).

`ptowsp_cuda_paged_decode_noalloc` is for callers that must not let a library
allocate device memory during a call -- serving engines whose memory is fully
reserved up front by their own KV-cache pool, or hosts that cannot take the
synchronisation cudaMalloc/cudaFree can cause.  It keeps its scratch in one
fixed array of device memory owned by the library.

This test calls it through the C ABI twice in a row (the second call with other
lengths, so stale scratch from the first call would show) and checks each
result against the regular entry point (`ptowsp_cuda_main` on the decode plan)
with the decode tests' tolerance.  It also checks that the second call takes no
device memory, and that a workload too big for the fixed array is refused.
The file name makes pytest collect it last.
"""

import ctypes as C

import numpy as np
import pytest

from pto_wsp_b200 import workloads
from pto_wsp_b200.runtime import CudaExecutable, load_library

pytestmark = pytest.mark.gpu


def check(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.sqrt(np.mean(ref * ref)) + 1e-12
    assert np.all(np.abs(got - ref) <= 2e-3 * (np.abs(ref) + scale))


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


def test_noalloc_matches_regular_entry_point_twice(require_cuda):
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
    check(d1[5].cpu().numpy(), run_regular(plan1, a1, R))

    d2 = to_device(torch, a2)  # inputs of the second call are allocated by the test, before measuring
    free_before = torch.cuda.mem_get_info()[0]
    rc = call_noalloc(f, torch, d2, R)
    free_after = torch.cuda.mem_get_info()[0]
    assert rc == 0, lib.ptowsp_cuda_last_error()
    assert free_after == free_before  # the call itself took no device memory
    out2 = d2[5].cpu().numpy()
    check(out2, run_regular(plan2, a2, R))
    assert not np.isnan(out2.astype(np.float32)).any()


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
