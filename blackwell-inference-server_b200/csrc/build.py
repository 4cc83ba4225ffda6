"""Build libbw_ops.so (sm_100a) in-tree.

    python blackwell-inference-server_b200/csrc/build.py [--verbose]

Compiles every ``*.cu`` here with nvcc for ``-gencode arch=compute_100a,code=sm_100a``
(relocatable device code, so the kernels share one device status word), links
them into ``blackwell_ops/_lib/libbw_ops.so`` next to the Python package, and
skips objects whose sources and headers are unchanged.  No ``--use_fast_math``:
the quantiser and merge must use IEEE division and round-to-nearest-even.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent / "blackwell_ops"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libbw_ops.so"
OBJ_DIR = CSRC / "_build"
INCLUDE = CSRC.parent.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC,-O2", "-I", str(INCLUDE)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *_deps()])


def build(verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    OBJ_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    cc = nvcc()
    sources = sorted(CSRC.glob("*.cu"))
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []

    def compile_one(src: Path):
        obj = OBJ_DIR / (src.stem + ".o")
        if not _stale(obj, src) and not ptxas_verbose:
            return obj, ""
        cmd = [cc, *ARCH, *CFLAGS, *extra, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        return obj, r.stderr

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, sources))
    objs = [o for o, _ in results]
    if ptxas_verbose:
        for _, log in results:
            sys.stderr.write(log)
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [cc, *ARCH, "-shared", "-rdc=true", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(LIB)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers / spills / smem per kernel")
    a = ap.parse_args()
    print(build(a.verbose, a.ptxas_verbose))
