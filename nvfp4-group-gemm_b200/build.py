"""Ahead-of-time build of the CUDA library for sm_100a.

The library is compiled in-tree with nvcc (``libnvfp4_group_gemm.so`` next to
this file) so that it travels with the source tree; no JIT cache is used.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_NAME = "libnvfp4_group_gemm.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
SOURCES = ["nvfp4_group_gemm.cu", "moe_host.cu", "ep_host.cu"]
HEADERS = ["grouped_gemm_kernel.cuh", "grouped_gemm_pair_kernel.cuh", "grouped_gemm_swap_kernel.cuh",
           "quantize_kernel.cuh", "moe_kernels.cuh", "nvfp4_quant_math.cuh", "ep_kernels.cuh",
           "row_ops.cuh", "host_common.cuh",
           "nvfp4_types.cuh", "sm100_ptx.cuh"]
PUBLIC_HEADER = os.path.join(os.path.dirname(HERE), "include", "nvfp4_group_gemm.h")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-shared",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or add /usr/local/cuda/bin to PATH)")


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    lib_t = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [PUBLIC_HEADER]
    return any(os.path.getmtime(d) > lib_t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; return its path."""
    if not force and not _stale():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", tmp, *[os.path.join(CSRC, s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
