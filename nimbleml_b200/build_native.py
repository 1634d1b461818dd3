"""Build step for the sm_100a C-ABI library ``_lib/libnimbleml_tied_ce.so``.

The library is compiled in-tree with nvcc for ``sm_100a`` only (tcgen05 /
TMA code has no portable fallback), linked against the static CUDA runtime,
and resolves the driver's ``cuTensorMapEncodeTiled`` at run time, so the .so
loads on hosts without a GPU. Run ``python -m nimbleml_b200.build_native``.

The same step builds ``_lib/nimbleml_tied_ce_native*.so``, the pybind11
module with the reference-style ``*_device`` entry points
(``csrc/tied_ce_pybind.cpp``), linked against the library with an
``$ORIGIN`` run path.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libnimbleml_tied_ce.so"
SOURCES = [CSRC / "tied_ce.cu", CSRC / "rowwise.cu"]
HEADERS = [CSRC / "sm100_ptx.cuh", CSRC / "common.cuh", REPO_DIR / "include" / "nimbleml_tied_ce.h"]
PYBIND_SOURCE = CSRC / "tied_ce_pybind.cpp"

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


def pybind_module_path() -> Path:
    ext = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return LIB_DIR / f"nimbleml_tied_ce_native{ext}"


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    built = target.stat().st_mtime
    return any(p.stat().st_mtime > built for p in deps)


def build_pybind(force: bool = False, verbose: bool = False) -> Path:
    """Compile the pybind11 module (g++) if it is older than its source or the library."""
    out = pybind_module_path()
    if not force and not _stale(out, [PYBIND_SOURCE, LIB_PATH, HEADERS[-1]]):
        return out
    import pybind11

    tmp = out.with_suffix(".tmp")
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           "-I", pybind11.get_include(), "-I", sysconfig.get_paths()["include"], "-I", str(REPO_DIR / "include"),
           str(PYBIND_SOURCE), "-L", str(LIB_DIR), "-l:" + LIB_PATH.name, "-Wl,-rpath,$ORIGIN", "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if a source is newer than the .so (or ``force``), then the pybind11 module."""
    if force or _stale(LIB_PATH, SOURCES + HEADERS):
        LIB_DIR.mkdir(parents=True, exist_ok=True)
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [_nvcc(), *NVCC_FLAGS, "-I", str(REPO_DIR / "include"), "-o", str(tmp), *map(str, SOURCES)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB_PATH)
    build_pybind(force=force, verbose=verbose)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
