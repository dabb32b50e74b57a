"""Builds libsandmuon_b200.so for sm_100a with nvcc, in-tree.

Usage:  python -m sandmuon_b200.csrc.build   (or sandmuon_b200.csrc.build.build())

The shared library lands next to the package (sandmuon_b200/libsandmuon_b200.so)
so it travels with the source tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PACKAGE = CSRC.parent
ROOT = PACKAGE.parent
LIB_NAME = "libsandmuon_b200.so"
LIB_PATH = PACKAGE / LIB_NAME
SOURCES = [CSRC / "libsandmuon_b200.cu"]
DEPENDS = SOURCES + [CSRC / "sm_common.cuh", CSRC / "sm_gemm.cuh", CSRC / "sm_kernels.cuh",
                     ROOT / "include" / "sandmuon_b200.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-warn-spills",
]


def nvcc_path() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the sandmuon_b200 CUDA library cannot be built")


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    built = LIB_PATH.stat().st_mtime
    return all(dep.stat().st_mtime <= built for dep in DEPENDS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles the library unless it is newer than every source file."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", str(ROOT / "include"), "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    if verbose and (result.stdout or result.stderr):
        print(result.stdout + result.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
