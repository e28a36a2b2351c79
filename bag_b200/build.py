"""Build ``libbag_b200.so`` in-tree with nvcc for sm_100a.

The CMake package (``CMakeLists.txt`` at the repository root) builds the same
sources as target ``bag::capi``; this script is the dependency-free path used
by the Python package and the test harness.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libbag_b200.so")
SOURCES = ["bag_kernels.cu", "bag_ws_kernel.cu", "bag_tc_kernel.cu", "bag_tc3_kernel.cu",
           "bag_capi.cu", "bag_noalloc.cu"]
HEADERS = ["bag_kernels.h", "bag_plan.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr"]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _inputs() -> list[str]:
    files = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    files.append(os.path.join(ROOT, "include", "bag_capi.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every CUDA source for sm_100a into ``bag_b200/libbag_b200.so``."""
    if not force and up_to_date():
        return LIB
    objs = []
    build_dir = os.path.join(HERE, "_build")
    os.makedirs(build_dir, exist_ok=True)
    for src in SOURCES:
        obj = os.path.join(build_dir, src.replace(".cu", ".o"))
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-c",
               os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        objs.append(obj)
    tmp = LIB + ".tmp"
    subprocess.check_call([nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
