"""Build libzs.so (all sm_100a kernels + the C ABI) in-tree with nvcc.

The library is a plain shared object: no torch headers, no Python API.  It is
written next to this file so it travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
LIB = PKG / "libzs.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the zs CUDA library cannot be built")
    return cand


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "zs.h"]


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), "-o", str(tmp), str(CSRC / "zs_lib.cu")]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose=True)
    print(LIB)
