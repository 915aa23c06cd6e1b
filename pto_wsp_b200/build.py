"""Build the native library ``pto_wsp_b200/lib/libptowsp_cuda.so`` in-tree.

Host C++ goes through nvcc's host compiler, CUDA sources are compiled for
``sm_100a`` only (``-gencode arch=compute_100a,code=sm_100a``), and the CUDA
runtime is linked statically so the library has no dependency on a particular
``libcudart`` at load time.  Incremental: an object is rebuilt when its source
or any header in ``csrc/`` is newer.

    python -m pto_wsp_b200.build [-v] [--force]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "lib" / "libptowsp_cuda.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
HOST_CXX = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else (shutil.which("g++") or "g++")


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or install the CUDA toolkit)")


def _sources() -> list[Path]:
    return sorted(p for p in CSRC.iterdir() if p.suffix in (".cpp", ".cu"))


def _headers_mtime() -> float:
    hs = [p for p in CSRC.iterdir() if p.suffix in (".hpp", ".cuh", ".h")]
    hs += list(INCLUDE.glob("*.h"))
    return max((p.stat().st_mtime for p in hs), default=0.0)


def _compile(src: Path, verbose: bool) -> Path:
    out = OBJ / (src.name + ".o")
    common = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "-ccbin", HOST_CXX, f"-I{INCLUDE}", f"-I{CSRC}"]
    if src.suffix == ".cu":
        cmd = [nvcc(), *ARCH, "-lineinfo", "--expt-relaxed-constexpr", *common, "-c", str(src), "-o", str(out)]
    else:
        cmd = [nvcc(), "-x", "cu", *ARCH, *common, "-c", str(src), "-o", str(out)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src.name}\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, file=sys.stderr)
    return out


def build(verbose: bool = False, force: bool = False, jobs: int | None = None) -> Path:
    OBJ.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    todo = []
    objs = []
    for src in _sources():
        out = OBJ / (src.name + ".o")
        objs.append(out)
        if force or not out.exists() or out.stat().st_mtime < max(src.stat().st_mtime, hdr):
            todo.append(src)
    # drop objects of deleted sources
    for stale in OBJ.glob("*.o"):
        if stale not in objs:
            stale.unlink()
    if todo:
        with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            list(ex.map(lambda s: _compile(s, verbose), todo))
    if todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-ccbin", HOST_CXX, "-cudart", "static", "-o", str(tmp), *map(str, objs),
               "-Xlinker", "--no-undefined", "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))


if __name__ == "__main__":
    main()
