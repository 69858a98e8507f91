"""Build libdflash_b200.so in-tree with nvcc for sm_100a.

The library is one translation unit (``csrc/dflash_b200.cu``) linked against
the static CUDA runtime; it resolves driver entry points at run time, so it
loads on machines without a GPU or libcuda.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
LIB_NAME = "libdflash_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME
INCLUDE_DIR = PKG_DIR.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2",
    "-shared",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build dflash-b200")


def sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh"))) + [INCLUDE_DIR / "dflash_b200.h"]


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile the library if any source is newer than the built .so."""
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", str(INCLUDE_DIR)]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    cmd += ["-o", str(tmp), str(CSRC / "dflash_b200.cu")]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose or ptxas_info:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="-v" in sys.argv)
    print(LIB_PATH)
