"""A generic kernel that contracts first and finishes row-locally (-m gpu): the f16 x f16 -> f32 matmul runs on the
tcgen05 tile kernel into scratch, the rest (column broadcast, scalar op, row max, row broadcast, exp) as one fused row
program; results against the oracle within the fp16-contraction tolerance, the makespan exact."""

import numpy as np
import pytest
from _mm_epilogue import mm_epilogue_arrays, mm_epilogue_plan
from cpu_sim import CpuSim

from pto_wsp_b200.runtime import CudaExecutable

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch,m,n,k,tn,op", [(2, 256, 512, 256, 256, "Sub"), (1, 128, 256, 2048, 256, "Sub"),
                                               (2, 256, 256, 512, 128, "Add")])
def test_matmul_epilogue_matches_oracle(batch, m, n, k, tn, op, require_cuda):
    rng = np.random.default_rng(m + n + k)
    plan = mm_epilogue_plan(batch, m, n, k, tn=tn, bias_op=op)
    (A, B, bias, C), views = mm_epilogue_arrays(rng, batch, m, n, k, tn=tn)
    ref_views = [v.copy() if i < 3 else v for i, v in enumerate(views)]
    C_ref = np.full_like(C, np.nan)
    ref_views[3] = C_ref.reshape(batch, m // 128, 128, n // tn, tn).transpose(0, 1, 3, 2, 4)
    cyc = CpuSim(plan).run(ref_views)
    ex = CudaExecutable(plan)
    assert ex.describe()["kernels"][0]["impl"] == "matmul_tcgen05+row_program"
    for _ in range(2):  # the second run replays the cached task table and stage records
        C[...] = np.nan
        assert ex.run_with_symbols(views, {}, {}, {}) == cyc
        np.testing.assert_allclose(C, C_ref, rtol=2e-3, atol=1e-6)
    assert ex.timing()["launches"] == 2  # the matmul and the fused epilogue
