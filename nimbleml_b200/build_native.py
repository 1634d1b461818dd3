"""Build step for the sm_100a C-ABI library ``_lib/libnimbleml_tied_ce.so``.

The library is compiled in-tree with nvcc for ``sm_100a`` only (tcgen05 /
TMA code has no portable fallback), linked against the static CUDA runtime,
and resolves the driver's ``cuTensorMapEncodeTiled`` at run time, so the .so
loads on hosts without a GPU. Run ``python -m nimbleml_b200.build_native``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libnimbleml_tied_ce.so"
SOURCES = [CSRC / "tied_ce.cu", CSRC / "rowwise.cu"]
HEADERS = [CSRC / "sm100_ptx.cuh", CSRC / "common.cuh", REPO_DIR / "include" / "nimbleml_tied_ce.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-cudart", "static",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > built for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if a source is newer than the .so (or ``force``)."""
    if not force and not _stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", str(REPO_DIR / "include"), "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
