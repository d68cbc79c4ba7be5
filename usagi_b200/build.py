"""Ahead-of-time build of the sm_100a kernel library (``libbsattn.so``, in-tree).

The reference JIT-compiled Triton variants at first call and precompiled stride classes in
``setup()`` (kernels/v4_leaderboard_0740ms.py:189-238).  Here the CUDA source is compiled once,
for sm_100a only, with nvcc; the CUDA runtime is linked statically and the driver entry point
for TMA descriptors is resolved at run time, so the library loads on hosts without a GPU.

Usage: ``python -m usagi_b200.build [--force]``
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
LIB_NAME = "libbsattn.so"
LIB_PATH = PKG_DIR / LIB_NAME

SOURCES = ["bsattn_fwd.cu", "csr_build.cu"]
HEADERS = ["sm100_ptx.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-cudart", "static",
    "-shared",
]


def _nvcc() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the sm_100a kernel library cannot be built")


def _inputs():
    files = [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [INCLUDE / "bsattn.h"]
    return files


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(f.stat().st_mtime > t for f in _inputs())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile ``csrc/*.cu`` into ``usagi_b200/libbsattn.so``; returns the library path."""
    if not force and not needs_build():
        return LIB_PATH
    cmd = [_nvcc(), *NVCC_FLAGS]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd += ["-o", str(tmp)] + [str(CSRC / s) for s in SOURCES]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose or ptxas_info:
        sys.stdout.write(res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB_PATH)
