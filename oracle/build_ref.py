#!/usr/bin/env python3
"""Compile the reference's header-only CUDA BAG into ``oracle/_ref/libbagref.so``.

The recipe compiles ``oracle/ref_harness.cu`` (a thin C-ABI wrapper) with
``-I <reference>/include``, so every kernel in the library is the reference's
own code, unmodified, built for sm_100a.  Output goes only to ``oracle/_ref/``
(git-ignored; it travels to the GPU box as a built file).  Needs the
reference checkout (its root given as an argument or by BAG_REFERENCE_ROOT), so
it runs only where that exists; elsewhere the prebuilt library is used as is.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libbagref.so")


def build(reference: str | None = None, force: bool = False) -> str | None:
    reference = reference or os.environ.get("BAG_REFERENCE_ROOT")
    src = os.path.join(HERE, "ref_harness.cu")
    include = os.path.join(reference, "include") if reference else None
    if not include or not os.path.isdir(include):
        return LIB if os.path.exists(LIB) else None
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(src):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    tmp = LIB + ".tmp"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
           "-Xcompiler", "-fPIC", "-shared", "-w", "-I", include, src, "-o", tmp, "-lcudart"]
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, force="--force" in sys.argv))
