"""Element-wise tolerance checks shared by the GPU parity tests.

north_star bars: fp32 row ops within 1e-5 relative; f16 contractions within 2e-3 relative of an fp64 recompute.
`assert_rel` applies a bar as a plain relative error on every element whose reference magnitude is at least
`floor`; elements below the floor (values that cancel to near zero, where a relative error has no meaning) are
held to the bar times the floor as an absolute error.
"""

from __future__ import annotations

import numpy as np

RTOL_ROWS = 1e-5      # fp32 row ops
RTOL_F16_MMA = 2e-3   # f16 contractions and f16 outputs, against fp64


def assert_rel(got, ref, rtol: float, floor: float) -> float:
    """Assert |got - ref| <= rtol * |ref| where |ref| >= floor, and <= rtol * floor elsewhere; return the worst
    relative error above the floor."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape
    assert not np.isnan(got).any(), "NaN in the result"
    err = np.abs(got - ref)
    big = np.abs(ref) >= floor
    rel = err[big] / np.abs(ref[big]) if big.any() else np.zeros(1)
    worst = float(rel.max()) if rel.size else 0.0
    assert worst <= rtol, f"relative error {worst:.3g} > {rtol:g} (floor {floor:.3g})"
    small = err[~big]
    if small.size:
        assert float(small.max()) <= rtol * floor, f"absolute error {float(small.max()):.3g} below the floor"
    return worst


def rms(a) -> float:
    a = np.asarray(a, np.float64)
    return float(np.sqrt(np.mean(a * a))) if a.size else 0.0
