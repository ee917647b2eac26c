"""Build the sm_100a CUDA library ``libmoe_b200.so`` in-tree.

Run ``python -m muxi_race_b200.build`` (or call :func:`build_library`). nvcc cross-compiles for
sm_100a without a GPU present. The library is placed next to this file so that it travels with
the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_NAME = "libmoe_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
SOURCES = ["moe_capi.cu"]
HEADERS = ["moe_gemm.cuh", "moe_gemm_pair.cuh", "moe_gemm_tn.cuh", "ep_p2p.cuh", "route_align.cuh", "router_topk.cuh", "ordered_combine.cuh", "gather_quant.cuh", "ep_kernels.cuh", "sm100_ptx.cuh"]
GENCODE = "arch=compute_100a,code=sm_100a"


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin directory on PATH")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_library(force: bool = False, verbose: bool = False) -> str:
    """Compile ``csrc/*.cu`` into ``libmoe_b200.so`` (skipped when up to date)."""
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(os.path.dirname(PKG_DIR), "include", "moe_b200.h"))
    if not force and not _stale(LIB_PATH, deps):
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [
        nvcc_path(), "-gencode", GENCODE, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
        "-Xcompiler", "-fvisibility=hidden", "-shared", "-o", tmp,
    ] + [os.path.join(CSRC, f) for f in SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose="-v" in sys.argv))
