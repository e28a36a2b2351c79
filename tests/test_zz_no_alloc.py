"""bag_sgemm_noalloc, the entry point for callers that cannot allocate device
memory (a framework or serving process that owns a fixed device-memory pool,
or a latency-critical caller that cannot let a library call cudaMalloc).

It must give the same result as the workspace entry point bag_sgemm_ex, call
after call, while using only its built-in 16 MiB scratch array, and must
refuse problems that need more scratch than that.  This file is collected
last so a stop-at-first-failure run has already run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROW_MAJOR = 1


def _rel(got, ref) -> float:
    import torch
    d = got.double() - ref.double()
    return float(torch.linalg.vector_norm(d) / torch.linalg.vector_norm(ref.double()))


def _noalloc(bag, a, b, c, depth, basis, beta=0.0) -> int:
    n_rows, k = a.shape
    n = b.shape[1]
    return bag.lib().bag_sgemm_noalloc(ROW_MAJOR, n_rows, n, k, a.data_ptr(), k, b.data_ptr(), n,
                                       c.data_ptr(), n, beta, depth, bag.BASIS[basis],
                                       ctypes.c_void_p(0))


@pytest.mark.parametrize("n,depth,basis", [(1024, 2, "minimal"), (768, 1, "full"),
                                           (1000, 2, "minimal")])
def test_noalloc_matches_workspace_entry_point(bag, cuda, n, depth, basis):
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device="cuda").manual_seed(n + depth)
    a = torch.randn(n, n, device="cuda", generator=g)
    b = torch.randn(n, n, device="cuda", generator=g)
    # The existing entry point, with a workspace the caller allocated.
    ws = bag.Workspace.for_problem(n, n, n, depth, basis)
    c_ref = torch.empty(n, n, device="cuda")
    bag.sgemm(a, b, c_ref, beta=0.0, depth=depth, basis=basis, workspace=ws)
    exact = a.double() @ b.double()
    torch.cuda.synchronize()
    for call in range(2):   # the second call sees the first call's scratch contents
        c = torch.full((n, n), float("nan"), device="cuda")
        torch.cuda.synchronize()
        allocs_before = bag.device_allocations()
        free_before = torch.cuda.mem_get_info()[0]
        status = _noalloc(bag, a, b, c, depth, basis)
        torch.cuda.synchronize()
        assert status == 0, bag.lib().bag_last_error()
        assert bag.device_allocations() == allocs_before   # the library allocated nothing
        if call == 1:   # after the first call set the device up, device memory is unchanged
            assert torch.cuda.mem_get_info()[0] == free_before
        assert bool(torch.isfinite(c).all())
        assert _rel(c, c_ref) <= 2e-6, (call, _rel(c, c_ref))
        assert _rel(c, exact) <= 1e-5


def test_noalloc_accumulates_with_beta_one(bag, cuda):
    import torch
    n = 512
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(n, n, device="cuda", generator=g)
    b = torch.randn(n, n, device="cuda", generator=g)
    c0 = torch.randn(n, n, device="cuda", generator=g)
    c = c0.clone()
    assert _noalloc(bag, a, b, c, 2, "minimal", beta=1.0) == 0
    assert _noalloc(bag, a, b, c, 2, "minimal", beta=1.0) == 0
    torch.cuda.synchronize()
    assert _rel(c, c0.double() + 2 * (a.double() @ b.double())) <= 1e-5


def test_noalloc_rejects_problems_beyond_its_scratch(bag, cuda):
    import torch
    n = 4096   # depth 2 needs 8 x 2048^2 floats, beyond the 4,194,304 built in
    a = torch.zeros(n, n, device="cuda")
    c = torch.full((n, n), 3.0, device="cuda")
    status = _noalloc(bag, a, a, c, 2, "minimal")
    assert status == 3   # BAG_ERR_WORKSPACE
    assert b"scratch" in bag.lib().bag_last_error()
    torch.cuda.synchronize()
    assert bool((c == 3.0).all())   # nothing was enqueued
    assert np.isclose(float(c[0, 0]), 3.0)


# 3xTF32 mode: a plan whose prepared TF32 operands fit in the built-in scratch
# runs on them (the CTA-pair leaf kernel); one whose operands do not fit runs
# the tensor kernel with the transforms fused in.  Both against the workspace
# entry point in the same mode, and within 1.25x the FFMA path's error (the
# reference's numerics) as the other 3xTF32 tests bound it.
@pytest.mark.parametrize("m,k,n,depth,kernel", [(512, 1024, 512, 0, "tf32_pair"),
                                                (512, 2048, 512, 1, "tf32_fused")])
def test_noalloc_in_3xtf32_mode(bag, cuda, m, k, n, depth, kernel):
    import torch
    g = torch.Generator(device="cuda").manual_seed(m + k + depth)
    a = torch.randn(m, k, device="cuda", generator=g)
    b = torch.randn(k, n, device="cuda", generator=g)
    exact = a.double() @ b.double()
    c_ffma = torch.empty(m, n, device="cuda")
    bag.sgemm(a, b, c_ffma, beta=0.0, depth=depth, workspace=bag.Workspace.for_problem(n, m, k, depth))
    bag.set_math_mode("3xtf32")
    try:
        ws = bag.Workspace.for_problem(n, m, k, depth)
        c_ref = torch.empty(m, n, device="cuda")
        bag.sgemm(a, b, c_ref, beta=0.0, depth=depth, workspace=ws)
        for call in range(2):
            c = torch.full((m, n), float("nan"), device="cuda")
            torch.cuda.synchronize()
            allocs = bag.device_allocations()
            assert _noalloc(bag, a, b, c, depth, "minimal") == 0, bag.lib().bag_last_error()
            torch.cuda.synchronize()
            assert bag.device_allocations() == allocs
            assert bag.last_leaf_kernel() == kernel, (call, bag.last_leaf_kernel())
            assert bool(torch.isfinite(c).all())
            assert _rel(c, exact) <= 1.25 * _rel(c_ffma, exact), call
            assert _rel(c, c_ref) <= 2e-6, call
    finally:
        bag.set_math_mode("ffma")
    assert bag.device_error() == 0
