"""Build libdimmerkv.so (sm_100a) in-tree with nvcc.

    python dimmer-kv_b200/build_lib.py [--verbose]

Objects go to dimmer-kv_b200/_build/, the library to dimmer-kv_b200/dimmerkv/_lib/libdimmerkv.so.
Sources are recompiled only when they (or a header) are newer than their object.
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
BUILD = PKG / "_build"
LIB = PKG / "dimmerkv" / "_lib" / "libdimmerkv.so"
INCLUDE = PKG.parent / "include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-I", str(INCLUDE)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or add CUDA to PATH")


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    newest_header = max((h.stat().st_mtime for h in headers), default=0.0)
    sources = sorted(CSRC.glob("*.cu"))
    compiler = nvcc()

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header):
            return obj
        cmd = [compiler, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stderr}")
        if verbose and res.stderr:
            print(res.stderr, file=sys.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objects = list(pool.map(compile_one, sources))
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objects):
        cmd = [compiler, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objects)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    args = parser.parse_args()
    print(build(args.verbose))
