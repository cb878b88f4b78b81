"""Build the native backend in-tree: ``metellus_b200/_lib/libmetellus_cuda.so``.

Run as ``python -m metellus_b200.csrc.build``. Uses nvcc for sm_100a; the library
links the CUDA runtime statically and NVRTC dynamically (rpath to the CUDA toolkit),
and resolves driver entry points at run time so it also loads on a machine without
a GPU driver (the CPU test suite checks its exported symbols there).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
REPO = PKG.parent
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libmetellus_cuda.so"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    exe = shutil.which("nvcc") or str(CUDA_HOME / "bin" / "nvcc")
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return exe


def build_backend(force: bool = False, verbose: bool = False) -> Path:
    src = PKG / "csrc" / "cuda_backend.cu"
    hdr = REPO / "include" / "metellus_b200.h"
    LIB_DIR.mkdir(exist_ok=True)
    if not force and LIB.exists() and LIB.stat().st_mtime >= max(src.stat().st_mtime, hdr.stat().st_mtime):
        return LIB
    cmd = [
        nvcc(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
        "-I", str(REPO / "include"), "-o", str(LIB), str(src),
        "-cudart", "static", "-L", str(CUDA_HOME / "lib64"), "-lnvrtc",
        f"-Xlinker=-rpath,{CUDA_HOME / 'lib64'}",
    ]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build_backend(force="--force" in sys.argv, verbose=True)
    print(LIB)
