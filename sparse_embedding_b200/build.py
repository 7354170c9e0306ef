"""Build recipe of the native library (libse_gpu.so, sm_100a).

    python -m sparse_embedding_b200.build

compiles the CUDA sources under csrc/ with nvcc for sm_100a into
sparse_embedding_b200/_lib/libse_gpu.so. The library links the CUDA runtime
statically, so it only needs the driver at run time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libse_gpu.so"
SOURCES = ["se_store.cu", "se_partition.cu", "se_unique.cu"]
HEADERS = ["se_common.cuh", "se_host.hpp", "se_store_kernels.cuh", "se_partition.cuh", "se_exchange.cuh",
           "se_accum.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    # Products and sums round separately unless a kernel asks for a fused
    # multiply-add; IEEE division and square root (no fast math).
    "--fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
    "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libse_gpu.so")
    return exe


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [PKG_DIR.parent / "include" / "se_gpu.h"]
    return any(d.stat().st_mtime > built for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(tmp), *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
