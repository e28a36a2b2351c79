"""This build against the reference's own CUDA BAG kernel on the same box.

The reference (`bag_cuda::matmul`, ColumnTile8 backend, Batched schedule,
Minimal basis) is compiled unmodified from its headers into
oracle/_ref/libbagref.so by oracle/build_ref.py.  Same N(0,1) inputs, depth 2,
CUDA-event timing after a warm-up; the tensor-core path must be faster and
within the error bound (<= 1.25x the reference's rel-F, <= 1e-4).  Run with
-s to see the measurements (one REFERENCE_SPEED line per size)."""

from __future__ import annotations

import ctypes
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libbagref.so")


def _ref():
    if not os.path.exists(REF_LIB):
        pytest.skip("reference CUDA library not built (oracle/build_ref.py)")
    lib = ctypes.CDLL(REF_LIB)
    lib.ref_bag_matmul.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 5 + [ctypes.c_void_p]
    lib.ref_last_error.restype = ctypes.c_char_p
    return lib


def _time(torch, fn, reps):
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


@pytest.mark.parametrize("n", [4096, 8192, 16384])
def test_faster_than_the_reference_bag_kernel(bag, cuda, n):
    import torch
    ref = _ref()
    depth, reps = 2, (3 if n < 16384 else 2)
    g = torch.Generator(device="cuda").manual_seed(n)
    a = torch.randn(n, n, device="cuda", generator=g)
    b = torch.randn(n, n, device="cuda", generator=g)
    stream = torch.cuda.current_stream().cuda_stream
    c_ref = torch.zeros(n, n, device="cuda")

    def run_ref():
        # Row-major C = A B is the column-major C^T = B^T A^T of the reference.
        status = ref.ref_bag_matmul(b.data_ptr(), a.data_ptr(), c_ref.data_ptr(), n, depth, 0, 2, 0,
                                    stream)
        assert status == 0, ref.ref_last_error()

    ms_ref = _time(torch, run_ref, reps)
    out = {"n": n, "depth": depth, "reference_cuda_bag_ms": ms_ref}
    for mode in ("ffma", "3xtf32"):
        bag.set_math_mode(mode)
        ws = bag.Workspace.for_problem(n, n, n, depth)
        c = torch.zeros(n, n, device="cuda")
        out[f"{mode}_ms"] = _time(torch, lambda: bag.sgemm(a, b, c, depth=depth, workspace=ws), reps)
        out[f"{mode}_path"] = bag.last_leaf_path()
        del ws
        torch.cuda.empty_cache()
    bag.set_math_mode("ffma")
    flops = 2.0 * n ** 3
    for key in ("reference_cuda_bag", "ffma", "3xtf32"):
        out[f"{key}_tflops"] = flops / (out[f"{key}_ms"] * 1e-3) / 1e12
    # Errors of one fresh call each (C starts at 0), against FP64 in column panels.
    c_ref.zero_()
    run_ref()
    bag.set_math_mode("3xtf32")
    ws = bag.Workspace.for_problem(n, n, n, depth)
    c_tc = torch.zeros(n, n, device="cuda")
    bag.sgemm(a, b, c_tc, beta=0.0, depth=depth, workspace=ws)
    bag.set_math_mode("ffma")
    torch.cuda.synchronize()
    num_r = num_t = den = 0.0
    a64 = a.double()
    for j in range(0, n, 4096):
        exact = a64 @ b[:, j:j + 4096].double()
        dr = c_ref[:, j:j + 4096].double() - exact
        dt = c_tc[:, j:j + 4096].double() - exact
        num_r += float((dr * dr).sum())
        num_t += float((dt * dt).sum())
        den += float((exact * exact).sum())
    out["reference_rel_f"] = (num_r / den) ** 0.5
    out["3xtf32_rel_f"] = (num_t / den) ** 0.5
    print("REFERENCE_SPEED " + json.dumps(out), flush=True)
    assert out["3xtf32_path"] == "3xtf32" and bag.device_error() == 0
    assert out["3xtf32_rel_f"] <= min(1.25 * out["reference_rel_f"], 1e-4)
    assert out["3xtf32_ms"] < out["reference_cuda_bag_ms"]
    assert np.isfinite(out["ffma_ms"])
