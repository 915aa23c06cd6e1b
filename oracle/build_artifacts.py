"""Build the reference's own CPU-sim artifacts of the five BASELINE configs (TEST / BASELINE INFRASTRUCTURE ONLY).

Each config's workload, written with the reference's unchanged Python API (tests/_frontend_workloads.py), is
lowered by the reference frontend (``workload_to_codegen_ir``) and compiled by the reference's own codegen
(``compile_codegen``, target ``cpu_sim``: ``src/python/pto_codegen.cpp:3352-3434``) into its CPU-sim artifact --
the generated ``<module>_main`` task loop plus one kernel per ``@kernel``, built by oracle/ref_compile.cpp against
the clean-room pto-isa stand-in (oracle/ptoisa).  The artifacts are written once per *unit* of the config (one
outer-axis element, or a 128-row slab for bgemm) to ``oracle/_ref/artifacts/config_<name>.so`` with a manifest;
``oracle/ref_runner.py`` runs them on the GPU box's host cores as ``bench.py --impl reference``.

Runs in the build container only (needs the reference checkout and oracle/_ref's module):

    PTOWSP_REFERENCE=<reference checkout> python oracle/build_artifacts.py
"""

from __future__ import annotations

import json
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
OUT = HERE / "_ref" / "artifacts"

# unit of each config: the workload arguments of tests/_frontend_workloads.py and how many units make the config
UNITS = {
    "softmax": {"fn": "softmax", "args": [1, 2048], "units": 32, "what": "one batch element: 2048 tiles of 32x256"},
    "rmsnorm": {"fn": "rmsnorm", "args": [1, 4096], "units": 64, "what": "one batch element: 4096 tiles of 16x128"},
    "bgemm": {"fn": "bgemm", "args": [1, 128, 2048, 2048], "units": 64 * 16,
              "what": "one 128-row slab of one batch element: 16 output tiles of 128x128, K = 2048"},
    "decode": {"fn": "decode", "args": [1, 8, 4, 128, 512, 512], "units": 64,
               "what": "one request x 8 kv heads (its pages renumbered; up to 512 pages = 8192 tokens)"},
    "indexer": {"fn": "indexer", "args": [1, 8, 64, 128, 32768, 2048], "units": 16,
                "what": "one batch element: 8 queries x 64 heads over 32768 keys, then top-2048 per query"},
}


def main() -> None:
    sys.path[:0] = [str(ROOT), str(HERE), str(ROOT / "tests")]
    from refpath import reference_root

    ref = reference_root()
    if ref is None:
        raise SystemExit("reference checkout not found: set PTOWSP_REFERENCE")
    sys.path[:0] = [str(HERE / "_ref"), str(ref / "python")]
    import _frontend_workloads as fw
    from pto_wsp.ir_bridge import cpp, workload_to_codegen_ir

    OUT.mkdir(parents=True, exist_ok=True)
    manifest = {}
    for name, u in UNITS.items():
        wl, tensors = getattr(fw, u["fn"])(*u["args"])
        build = workload_to_codegen_ir(wl, module_name=f"config_{name}")
        opts = cpp.CompileOptions()
        opts.target = "cpu_sim"
        res = cpp.compile_codegen(build.module, opts)
        so = OUT / f"config_{name}.so"
        shutil.copyfile(res["so_path"], so)
        manifest[name] = {"so": so.name, "entrypoint": str(res["entrypoint"]), "args": u["args"],
                          "units": u["units"], "what": u["what"],
                          "tensors": [{"shape": list(t.shape), "dtype": str(t.dtype.name).lower()} for t in tensors]}
        print(f"{name}: {so.name} ({res['entrypoint']})")
    (OUT / "manifest.json").write_text(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    main()
