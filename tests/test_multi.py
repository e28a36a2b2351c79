"""One process, several GPUs: bag_sgemm_multi (row/column-band shards moved by
peer copies).  CPU part: the device grid and argument checks; GPU part: the
same path on one GPU listed several times (every shard copy, band offset and
per-device workspace runs, peer copies become local ones) and, with two GPUs
present, across two devices -- each against FP64 and against the single-GPU
call."""

from __future__ import annotations

import pytest

import bag_b200 as bag


@pytest.mark.parametrize("ngpus,grid", [(1, (1, 1)), (2, (2, 1)), (3, (3, 1)), (4, (2, 2)),
                                        (8, (4, 2))])
def test_grid_matches_the_bench_grid(ngpus, grid):
    import bench
    assert bag.multi_grid(ngpus) == grid
    if ngpus in (1, 2, 4, 8):
        assert bench.shard_grid(ngpus) == grid


def test_bad_arguments_fail_before_any_device_work():
    with pytest.raises(ValueError):
        bag.MultiWorkspace([], 512, 512, 512)
    # A 2 x 1 grid at depth 1 needs M of the column-major problem -- N of the
    # row-major call -- divisible by 2 x 2 = 4.
    with pytest.raises(ValueError):
        bag.MultiWorkspace([0, 0], 512, 514, 512, depth=1)


def _rel(torch, c, a, b, c0=None):
    exact = a.double() @ b.double()
    if c0 is not None:
        exact = exact + c0.double()
    return float((c.double() - exact).norm() / exact.norm())


@pytest.mark.gpu
@pytest.mark.parametrize("devices,m,n,k,depth,math,beta", [
    ([0], 512, 512, 512, 1, "ffma", 0.0),
    ([0, 0], 1024, 512, 768, 1, "ffma", 1.0),
    ([0, 0, 0, 0], 2048, 2048, 2048, 2, "ffma", 0.0),
    ([0, 0, 0, 0, 0, 0, 0, 0], 4096, 4096, 4096, 2, "3xtf32", 1.0),
    ([0, 0], 2048, 4096, 4096, 1, "3xtf32", 0.0),
])
def test_multi_on_one_gpu(bag, cuda, devices, m, n, k, depth, math, beta):
    import torch
    g = torch.Generator(device="cuda").manual_seed(m + n + k + depth)
    a = torch.randn(m, k, device="cuda", generator=g)
    b = torch.randn(k, n, device="cuda", generator=g)
    c0 = torch.randn(m, n, device="cuda", generator=g)
    bag.set_math_mode(math)
    try:
        ws = bag.MultiWorkspace(devices, m, n, k, depth=depth)
        c = c0.clone()
        bag.sgemm_multi(a, b, c, ws, beta=beta)
        torch.cuda.synchronize()
        ref = c0.clone()
        wss = bag.Workspace.for_problem(n, m, k, depth)
        bag.sgemm(a, b, ref, beta=beta, depth=depth, workspace=wss)
        torch.cuda.synchronize()
    finally:
        bag.set_math_mode("ffma")
    assert bag.device_error() == 0
    base = c0 if beta else None
    err, err_single = _rel(torch, c, a, b, base), _rel(torch, ref, a, b, base)
    assert err <= 1.25 * err_single + 1e-9, (err, err_single)
    # Same leaves, same blocks: only the atomic accumulation order may differ.
    assert float((c - ref).double().norm() / ref.double().norm()) <= 1e-6


@pytest.mark.gpu
def test_multi_across_two_gpus(bag, cuda):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    m = n = k = 4096
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(m, k, device="cuda", generator=g)
    b = torch.randn(k, n, device="cuda", generator=g)
    bag.set_math_mode("3xtf32")
    try:
        ws = bag.MultiWorkspace([0, 1], m, n, k, depth=2)
        c = torch.zeros(m, n, device="cuda")
        bag.sgemm_multi(a, b, c, ws, beta=0.0)
        torch.cuda.synchronize()
        ref = torch.zeros(m, n, device="cuda")
        bag.sgemm(a, b, ref, beta=0.0, depth=2, workspace=bag.Workspace.for_problem(n, m, k, 2))
        torch.cuda.synchronize()
    finally:
        bag.set_math_mode("ffma")
    assert bag.device_error() == 0
    assert _rel(torch, c, a, b) <= 1.25 * _rel(torch, ref, a, b) + 1e-9
    assert float((c - ref).double().norm() / ref.double().norm()) <= 1e-6
