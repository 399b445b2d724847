"""Build libzimage_b200.so (sm_100a) in-tree with nvcc.

    python comfyui-zimage-triton_b200/csrc/build.py [--force] [--verbose]

Objects go to csrc/_build/, the shared library to zimage_b200/libzimage_b200.so.
Rebuilds only when a source or header is newer than the library.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent / "zimage_b200"
INCLUDE = CSRC.parent.parent / "include"
OUT = PKG / "libzimage_b200.so"
SOURCES = ["zib_api.cu", "rowops.cu", "gemm_w8a8.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return OUT
    bdir = CSRC / "_build"
    bdir.mkdir(exist_ok=True)
    objs = []
    for s in SOURCES:
        o = bdir / (Path(s).stem + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / s), "-o", str(o)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(o))
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs, "-lcudart_static",
           "-Xcompiler", "-fPIC"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
    sys.exit(0)
