"""Ahead-of-time build of the sm_100a kernel library (``libbsattn.so``, in-tree).

The reference JIT-compiled Triton variants at first call and precompiled stride classes in
``setup()`` (kernels/v4_leaderboard_0740ms.py:189-238).  Here the CUDA source is compiled once,
for sm_100a only, with nvcc; the CUDA runtime is linked statically and the driver entry point
for TMA descriptors is resolved at run time, so the library loads on hosts without a GPU.

Usage: ``python -m usagi_b200.build [--force]``
"""
from __future__ import annotations

import hashlib
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
# Hash of the sources, headers and flags the in-tree library was built from (written next to it).
STAMP_PATH = PKG_DIR / (LIB_NAME + ".sha256")

SOURCES = ["bsattn_fwd.cu", "csr_build.cu", "peer.cu"]
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


def source_hash() -> str:
    """sha256 over the compile flags and the bytes of every source and header of the library."""
    h = hashlib.sha256()
    h.update(" ".join(NVCC_FLAGS).encode())
    for f in _inputs():
        h.update(f.name.encode())
        h.update(f.read_bytes())
    return h.hexdigest()


def needs_build() -> bool:
    """True unless the in-tree library exists and its stamp names the current sources: a library
    built from other sources (whatever its file time) is rebuilt."""
    if not LIB_PATH.exists() or not STAMP_PATH.exists():
        return True
    return STAMP_PATH.read_text().strip() != source_hash()


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
    digest = source_hash()
    os.replace(tmp, LIB_PATH)
    STAMP_PATH.write_text(digest + "\n")
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB_PATH)
