"""Build ``libmcl4moe.so`` (the C-ABI library) in place with nvcc for sm_100a.

    python mcl4-coe_b200/build.py

The library is written next to this file so it travels with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libmcl4moe.so"
SOURCES = ["quant.cu", "router.cu", "route.cu", "gemm_fp4.cu", "api.cu", "noalloc.cu", "ep.cu", "peer.cu",
           "backward.cu", "wgrad.cu", "linear_bwd.cu"]
HEADERS = ["common.cuh", "kernels.cuh", "sr.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2",
    "-shared",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found (set NVCC or put CUDA's bin on PATH)")
    return cand


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    mtime = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [HERE.parent / "include" / "mcl4moe.h", Path(__file__)]
    return all(d.stat().st_mtime <= mtime for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(tmp), *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, cwd=str(CSRC), capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
