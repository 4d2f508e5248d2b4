"""Build the C-ABI shared library ``libflash_ulysses_b200.so`` in-tree.

Compiles ``csrc/*.cu`` for sm_100a with nvcc and links the CUDA runtime
statically, so the library depends only on the driver.  Usage::

    python -m flash_ulysses_b200.build [--verbose-ptxas]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB_NAME = "libflash_ulysses_b200.so"
LIB_PATH = PKG / LIB_NAME
SOURCES = ["fu_capi.cu", "fu_qkv.cu", "fu_oproj.cu"]
FAST_SOURCE = "fu_pyfast.cpp"
FAST_PATH = PKG / ("_fu_fast" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or add the CUDA toolkit to PATH")


def _stale():
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    deps += list(INCLUDE.glob("*.h"))
    return any(d.stat().st_mtime > built for d in deps)


def build_fast(force=False):
    """The CPython binding of the per-call entry point (links the library)."""
    src = CSRC / FAST_SOURCE
    if (not force and FAST_PATH.exists() and FAST_PATH.stat().st_mtime > LIB_PATH.stat().st_mtime
            and FAST_PATH.stat().st_mtime > src.stat().st_mtime):
        return FAST_PATH
    cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
    tmp = FAST_PATH.with_suffix(".tmp")
    cmd = [cxx, "-O2", "-shared", "-fPIC", "-std=c++17",
           "-I", sysconfig.get_paths()["include"], "-I", str(INCLUDE), str(src),
           "-L", str(PKG), "-l:" + LIB_NAME, "-Wl,-rpath,$ORIGIN", "-o", str(tmp)]
    subprocess.run(cmd, check=True)
    os.replace(tmp, FAST_PATH)
    return FAST_PATH


def build(force=False, verbose_ptxas=False):
    """Compile the library (and its CPython fast-call binding) if any source is
    newer than it; returns the library path."""
    if not force and not verbose_ptxas and not _stale():
        build_fast()
        return LIB_PATH
    nvcc = nvcc_path()
    cmd = [
        nvcc, *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-shared",
        "-Xcompiler", "-fPIC,-fvisibility=hidden", "-cudart", "static",
        "-Xlinker", "-soname," + LIB_NAME,
        "-I", str(INCLUDE), "-I", str(CSRC),
        "-DFU_BUILDING_LIBRARY",
    ]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd += [str(CSRC / s) for s in SOURCES] + ["-o", str(tmp)]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    build_fast(force=True)
    return LIB_PATH


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose_ptxas=args.verbose_ptxas)
    print(path)


if __name__ == "__main__":
    sys.exit(main())
