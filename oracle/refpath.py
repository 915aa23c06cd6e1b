"""Where the reference checkout is (TEST / FIXTURE INFRASTRUCTURE ONLY).

The reference sources are needed only to build its IR module into ``oracle/_ref`` and to regenerate the golden
fixtures; GPU runs never read them.  The location comes from the ``PTOWSP_REFERENCE`` environment variable, else a
checkout named ``reference`` beside this repository; ``None`` when neither holds the reference sources.
"""

from __future__ import annotations

import os
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
MARKER = Path("src") / "python" / "pto_codegen.cpp"


def reference_root() -> Path | None:
    env = os.environ.get("PTOWSP_REFERENCE")
    for cand in ([Path(env)] if env else []) + [ROOT.parent / "reference"]:
        if (cand / MARKER).is_file():
            return cand.resolve()
    return None
