"""Loader for tests/golden/ref_cases.{json,npz} (captured by tests/golden/make_golden.py)."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent / "golden"


def load_cases() -> list[dict]:
    return json.loads((HERE / "ref_cases.json").read_text())


_NPZ = None


def _npz():
    global _NPZ
    if _NPZ is None:
        _NPZ = dict(np.load(HERE / "ref_cases.npz"))
    return _NPZ


def case_index(cases: list[dict], name: str) -> int:
    return next(i for i, c in enumerate(cases) if c["name"] == name)


def materialize(case: dict, idx: int):
    """Fresh input buffers laid out exactly like the reference run's numpy views."""
    z = _npz()
    roots = []
    for i, r in enumerate(case["roots"]):
        raw = z[f"c{idx}_in{i}"].copy()
        roots.append(raw.view(np.dtype(r["dtype"])).reshape(r["shape"]))

    def view(d):
        root = roots[d["root"]]
        return np.ndarray(shape=tuple(d["shape"]), dtype=np.dtype(d["dtype"]), buffer=root,
                          offset=d["offset"], strides=tuple(d["strides"]))

    arrays = [view(d) for d in case["arrays"]]
    sptr = {int(d["id"]): view(d) for d in case["symbols_ptr"]}
    axis = dict(case["axis_sizes"])
    syms = {int(k): int(v) for k, v in case["symbols_u64"].items()}
    return roots, arrays, axis, syms, sptr


def expected_roots(case: dict, idx: int) -> list[np.ndarray]:
    z = _npz()
    return [z[f"c{idx}_out{i}"].view(np.dtype(r["dtype"])).reshape(r["shape"]) for i, r in enumerate(case["roots"])]


def artifact_roots(case: dict, idx: int) -> list[np.ndarray] | None:
    """Output buffers of the reference's own CPU-sim artifact on the same inputs (None for older fixtures)."""
    z = _npz()
    if f"c{idx}_art0" not in z:
        return None
    return [z[f"c{idx}_art{i}"].view(np.dtype(r["dtype"])).reshape(r["shape"]) for i, r in enumerate(case["roots"])]
