"""Shared test setup.

* ``gpu`` marks tests that need a CUDA device (run with ``-m gpu`` on a B200).
* The reference frontend (``pto_wsp`` + its ``pto_ir_cpp`` module) is only
  available in the build container (reference sources plus ``oracle/_ref``);
  tests that need it are skipped elsewhere.  GPU tests never need it.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

from refpath import reference_root  # noqa: E402

REF = reference_root()  # PTOWSP_REFERENCE, else a `reference` checkout beside the repo; None: tests skip


def reference_available() -> bool:
    ext = list((ROOT / "oracle" / "_ref").glob("pto_ir_cpp*.so"))
    return REF is not None and (REF / "python" / "pto_wsp").is_dir() and bool(ext)


def import_reference():
    """Put the reference frontend on sys.path (build container only)."""
    if not reference_available():
        pytest.skip("reference frontend not available (build container only)")
    for p in (str(ROOT / "oracle" / "_ref"), str(REF / "python")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import pto_wsp  # noqa: F401

    return pto_wsp


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def cuda_available() -> bool:
    try:
        from pto_wsp_b200.runtime import device_count

        return device_count() > 0
    except Exception:  # noqa: BLE001
        return False


@pytest.fixture(scope="session")
def require_cuda():
    if not cuda_available():
        pytest.skip("no CUDA device")
