"""Lightning indexer scoring + top-k (-m gpu).

Parity is split (scores are floating point, indices are not):
  (i)  GPU scores vs an fp64 recompute within 2e-3 relative;
  (ii) GPU top-k over the GPU's own score buffer == the oracle's stable
       selection (score desc, ties -> lower index) on that buffer, bit-exact;
  (iii) GPU indices vs the selection on the fp64 scores: an index may differ only where the two scores lie within
       the score tolerance of the K-th score (a near-tie resolved the other way);
  (iv) top-k kernel alone on adversarial rows (heavy ties, +-0, extremes), bit-exact.
"""

import numpy as np
import pytest
from cpu_sim import stable_topk

from pto_wsp_b200 import workloads
from pto_wsp_b200.runtime import CudaExecutable

pytestmark = pytest.mark.gpu


def scores64(q, k, w):
    B, QH, D = q.shape
    Q, H = w.shape[1], w.shape[2]
    out = np.empty((B, Q, k.shape[1]))
    for b in range(B):
        dots = (q[b].astype(np.float64) @ k[b].astype(np.float64).T).reshape(Q, H, -1)
        out[b] = np.einsum("qh,qht->qt", w[b].astype(np.float64), np.maximum(dots, 0))
    return out


def test_indexer_small_vs_fp64_and_topk_exact(require_cuda):
    rng = np.random.default_rng(0)
    plan, arrays = workloads.indexer_inputs(rng, 2, 1024, 64)
    ex = CudaExecutable(plan)
    assert [k["impl"] for k in ex.describe()["kernels"]] == ["lightning_indexer_score", "topk_select"]
    got = [a.copy() for a in arrays]
    ex.run_with_symbols(got, {}, {}, {})
    s, idx = got[3], got[4]
    ref = scores64(arrays[0], arrays[1], arrays[2])
    err = np.abs(s - ref) / (np.abs(ref) + np.sqrt(np.mean(ref * ref)))
    assert err.max() <= 2e-3, err.max()
    for b in range(2):
        for qq in range(8):
            assert idx[b, qq].tolist() == stable_topk(s[b, qq], 64).tolist()
            # (iii) against the fp64 scores: the chosen sets differ only by near-ties at the threshold
            ref_idx = stable_topk(ref[b, qq], 64)
            kth = np.sort(ref[b, qq])[::-1][63]
            tol = 2e-3 * (abs(kth) + np.sqrt(np.mean(ref[b, qq] ** 2)))
            for i in set(idx[b, qq].tolist()) ^ set(ref_idx.tolist()):
                assert abs(ref[b, qq, i] - kth) <= tol, (b, qq, i)


@pytest.mark.parametrize("kind", ["ties", "zeros", "mixed", "sorted", "reverse", "nan"])
def test_topk_adversarial_rows_bit_exact(kind, require_cuda):
    rng = np.random.default_rng(1)
    rows, n, k = 6, 4096, 2048
    if kind == "ties":
        s = rng.integers(0, 3, (rows, 1, n)).astype(np.float32)
    elif kind == "zeros":
        s = np.where(rng.random((rows, 1, n)) < 0.5, np.float32(0.0), np.float32(-0.0)).astype(np.float32)
        s[:, :, ::7] = 1.0
    elif kind == "mixed":
        s = rng.standard_normal((rows, 1, n)).astype(np.float32)
        s[:, :, ::5] = np.float32(3.4e38)
        s[:, :, 1::11] = -np.inf
        s[:, :, 2::13] = np.inf
    elif kind == "nan":
        s = rng.standard_normal((rows, 1, n)).astype(np.float32)
        s[:, :, ::9] = np.float32(np.nan)
        s[:, :, 4::17] = -np.float32(np.nan)
    elif kind == "sorted":
        s = np.tile(np.arange(n, dtype=np.float32), (rows, 1, 1))
    else:
        s = np.tile(np.arange(n, dtype=np.float32)[::-1].copy(), (rows, 1, 1))
    out = np.full((rows, 1, k), -7, np.int32)
    CudaExecutable(workloads.topk_plan(rows, n, k)).run_with_symbols([s, out], {}, {}, {})
    for r in range(rows):
        assert out[r, 0].tolist() == stable_topk(s[r, 0], k).tolist()


@pytest.mark.parametrize("kind", ["three_values", "top_half_equal", "narrow_band"])
def test_topk_wide_rows_with_many_candidates_bit_exact(kind, require_cuda):
    # more keys share the threshold's 16-bit prefix than the candidate list holds (it overflows to a row sweep),
    # and more keys equal the threshold than the pairwise tie ranking takes (an index-ordered sweep breaks them)
    rng = np.random.default_rng(11)
    rows, n, k = 3, 32768, 2048
    if kind == "three_values":
        s = rng.integers(0, 3, (rows, 1, n)).astype(np.float32)
    elif kind == "top_half_equal":
        s = rng.standard_normal((rows, 1, n)).astype(np.float32)
        s[:, :, rng.permutation(n)[: n // 2]] = 5.0
    else:  # distinct values inside one 16-bit key prefix: many candidates, no ties
        s = (1.0 + rng.permutation(n).astype(np.float32) * 2.0 ** -23).astype(np.float32).reshape(1, 1, n)
        s = np.repeat(s, rows, axis=0)
    out = np.full((rows, 1, k), -7, np.int32)
    CudaExecutable(workloads.topk_plan(rows, n, k)).run_with_symbols([s, out], {}, {}, {})
    for r in range(rows):
        assert out[r, 0].tolist() == stable_topk(s[r, 0], k).tolist()


@pytest.mark.parametrize("n,k", [(1, 1), (100, 7), (1000, 1000), (1025, 1), (5000, 33), (32768, 2048),
                                 (49152, 2048), (20000, 4096), (3000, 3000)])
def test_topk_sizes_bit_exact(n, k, require_cuda):
    rng = np.random.default_rng(n + k)
    rows = 3
    s = (rng.standard_normal((rows, 1, n)) * 10).astype(np.float16).astype(np.float32)  # f16 grid: many ties
    out = np.full((rows, 1, k), -7, np.int32)
    CudaExecutable(workloads.topk_plan(rows, n, k)).run_with_symbols([s, out], {}, {}, {})
    for r in range(rows):
        assert out[r, 0].tolist() == stable_topk(s[r, 0], k).tolist()


def test_indexer_config5_full_size(require_cuda):
    torch = pytest.importorskip("torch")
    B, T, K = 16, 32768, 2048
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    q = torch.randn((B, 512, 128), generator=g, device="cuda").half()
    k = torch.randn((B, T, 128), generator=g, device="cuda").half()
    w = torch.rand((B, 8, 64), generator=g, device="cuda")
    s = torch.full((B, 8, T), float("nan"), device="cuda")
    idx = torch.full((B, 8, K), -1, device="cuda", dtype=torch.int32)
    ex = CudaExecutable(workloads.indexer_plan(B, 8, 64, 128, T, K))
    ex.run_with_symbols([q, k, w, s, idx], {}, {}, {})
    s_h, idx_h = s.cpu().numpy(), idx.cpu().numpy()
    assert not np.isnan(s_h).any()
    for b in (0, 9, 15):
        ref = scores64(q[b:b + 1].cpu().numpy(), k[b:b + 1].cpu().numpy(), w[b:b + 1].cpu().numpy())[0]
        err = np.abs(s_h[b] - ref) / (np.abs(ref) + np.sqrt(np.mean(ref * ref)))
        assert err.max() <= 2e-3, err.max()
        for qq in range(8):  # (iii): against the fp64 selection, only near-ties at the threshold may differ
            kth = np.sort(ref[qq])[::-1][K - 1]
            tol = 2e-3 * (abs(kth) + np.sqrt(np.mean(ref[qq] ** 2)))
            diff = set(idx_h[b, qq].tolist()) ^ set(stable_topk(ref[qq], K).tolist())
            assert all(abs(ref[qq, i] - kth) <= tol for i in diff), (b, qq, len(diff))
    for b in range(B):
        for qq in range(8):
            assert idx_h[b, qq].tolist() == stable_topk(s_h[b, qq], K).tolist()
