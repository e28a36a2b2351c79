"""GPU tests of the 3xTF32 tcgen05 variant (bag_set_math_mode(BAG_MATH_3XTF32)).

Bar: relative Frobenius error vs FP64 no worse than 1.25x the FFMA path's (the
reference's numerics) on the same inputs, and <= 1e-4; ragged edges, K tails,
BAG depths and bases, batches; leaves shorter than K = 1024 stay on the FFMA
kernel; every in-kernel wait completes (device error word 0)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import bag_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture
def tensor_mode(bag, cuda):
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    bag.set_math_mode("3xtf32")
    yield bag
    bag.set_math_mode("ffma")


def _operands(torch, m, k, n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(m, k, device="cuda", generator=g),
            torch.randn(k, n, device="cuda", generator=g))


def _sgemm(bag, torch, a, b, depth, basis, ws, mode):
    bag.set_math_mode(mode)
    c = torch.zeros(a.shape[0], b.shape[1], device="cuda")
    bag.sgemm(a, b, c, beta=0.0, depth=depth, basis=basis, workspace=ws)
    torch.cuda.synchronize()
    return c, bag.last_leaf_path()


def _rel(torch, c, a, b):
    exact = a.double() @ b.double()
    return float((c.double() - exact).norm() / exact.norm())


# Leaf K >= 1024 everywhere: the tensor path runs.  Ragged M/N, a K tail that
# is not a multiple of the stage length, depths 0-2 and both bases.
@pytest.mark.parametrize("m,k,n,depth,basis", [
    (256, 1024, 384, 0, "minimal"), (200, 1032, 136, 0, "minimal"), (132, 1100, 260, 0, "minimal"),
    (2048, 2048, 2048, 1, "minimal"), (1536, 2064, 1032, 1, "minimal"),
    (2048, 2048, 2048, 1, "classic"), (4096, 4096, 4096, 2, "minimal"),
    (2048, 4096, 2048, 2, "classic"), (2048, 4096, 2048, 2, "full")])
def test_tensor_path_error(tensor_mode, m, k, n, depth, basis):
    import torch
    bag = tensor_mode
    a, b = _operands(torch, m, k, n, seed=m + k + n + depth)
    # sgemm's row-major call is the column-major C^T(n x m) = B^T A^T; leaf K = k / 2^depth.
    ws = bag.Workspace.for_problem(n, m, k, depth, basis) if depth >= 2 or basis != "minimal" else None
    c_tc, path = _sgemm(bag, torch, a, b, depth, basis, ws, "3xtf32")
    assert path == "3xtf32"
    assert bag.device_error() == 0
    c_ff, path_ff = _sgemm(bag, torch, a, b, depth, basis, ws, "ffma")
    assert path_ff == "ffma"
    err, ffma = _rel(torch, c_tc, a, b), _rel(torch, c_ff, a, b)
    assert err <= 1e-4
    assert err <= 1.25 * ffma, (err, ffma)


@pytest.mark.parametrize("m,k,n,depth", [(128, 8, 128, 0), (512, 256, 512, 0), (1024, 1024, 1024, 1),
                                         (768, 520, 1000, 1)])
def test_short_leaves_stay_on_ffma(tensor_mode, m, k, n, depth):
    import torch
    bag = tensor_mode
    a, b = _operands(torch, m, k, n, seed=7)
    c_tc, path = _sgemm(bag, torch, a, b, depth, "minimal", None, "3xtf32")
    assert path == "ffma"
    c_ff, _ = _sgemm(bag, torch, a, b, depth, "minimal", None, "ffma")
    if depth == 0:   # one writer per element: the same kernel gives the same bits
        assert torch.equal(c_tc, c_ff)
    assert bag.device_error() == 0


def test_tensor_path_accumulates(tensor_mode):
    import torch
    bag = tensor_mode
    n = 2048
    a, b = _operands(torch, n, n, n, seed=3)
    c0 = torch.randn(n, n, device="cuda")
    c = c0.clone()
    bag.sgemm(a, b, c, beta=1.0, depth=1)
    bag.sgemm(a, b, c, beta=1.0, depth=1)
    torch.cuda.synchronize()
    assert bag.last_leaf_path() == "3xtf32"
    exact = c0.double() + 2 * (a.double() @ b.double())
    assert float((c.double() - exact).norm() / exact.norm()) <= 2e-6
    assert bag.device_error() == 0


def test_tensor_path_batched(tensor_mode):
    import torch
    bag = tensor_mode
    batch, n = 3, 2048
    g = torch.Generator(device="cuda").manual_seed(4)
    a = torch.rand(batch, n, n, device="cuda", generator=g)
    b = torch.rand(batch, n, n, device="cuda", generator=g)
    c = torch.zeros(batch, n, n, device="cuda")
    bag.sgemm_batched(a, b, c, beta=0.0, depth=1)
    torch.cuda.synchronize()
    assert bag.last_leaf_path() == "3xtf32"
    exact = a.double() @ b.double()
    assert float((c.double() - exact).norm() / exact.norm()) <= 2e-6
    assert bag.device_error() == 0


def test_tensor_path_against_oracle(tensor_mode):
    """Against the restated reference numerics (sequential-fmaf leaves) on the
    same inputs: rectangular, one level, leaf K = 1024."""
    import torch
    bag = tensor_mode
    m, k, n = 512, 2048, 256
    rng = np.random.default_rng(9)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    tc = torch.zeros(m, n, device="cuda")
    bag.sgemm(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), tc, beta=0.0, depth=1)
    torch.cuda.synchronize()
    assert bag.last_leaf_path() == "3xtf32"
    got = tc.cpu().numpy()
    ref = O.bag_product(a, b, 1, "minimal", leaf="fmaf")
    exact = O.fp64_matmul(a, b)
    assert O.rel_frobenius(got, exact) <= 1.25 * O.rel_frobenius(ref, exact)
    assert bag.device_error() == 0


# Prepared-operand path: a workspace created in 3xTF32 mode also holds every
# leaf operand as TF32 hi/lo rows (one prepare pass, then TMA/SS-MMA leaves).
@pytest.mark.parametrize("m,k,n,depth,basis", [
    (512, 2048, 768, 0, "minimal"), (1032, 4096, 2056, 2, "minimal"),
    (4096, 4096, 4096, 2, "minimal"), (2048, 4096, 2048, 2, "full"),
    (2048, 2048, 2048, 1, "classic"), (1000, 2048, 1160, 1, "minimal"),
    (2048, 4096, 2048, 2, "winograd")])
def test_prepared_path(tensor_mode, m, k, n, depth, basis):
    import torch
    bag = tensor_mode
    a, b = _operands(torch, m, k, n, seed=m + n + depth)
    # Column-major problem of the row-major call: C^T(n x m) = B^T A^T.
    ws = bag.Workspace.for_problem(n, m, k, depth, basis)
    bag.set_math_mode("ffma")
    ws_ffma = bag.Workspace.for_problem(n, m, k, depth, basis)
    assert ws.bytes() > ws_ffma.bytes()   # the prepared region
    c_tc, path = _sgemm(bag, torch, a, b, depth, basis, ws, "3xtf32")
    assert path == "3xtf32"
    assert bag.device_error() == 0
    c_ff, _ = _sgemm(bag, torch, a, b, depth, basis, ws_ffma, "ffma")
    err, ffma = _rel(torch, c_tc, a, b), _rel(torch, c_ff, a, b)
    assert err <= 1e-4
    assert err <= 1.25 * ffma, (err, ffma)


def test_prepared_path_batched_and_accumulating(tensor_mode):
    import torch
    bag = tensor_mode
    batch, n = 2, 2048
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.rand(batch, n, n, device="cuda", generator=g)
    b = torch.rand(batch, n, n, device="cuda", generator=g)
    c0 = torch.rand(batch, n, n, device="cuda", generator=g)
    ws = bag.Workspace.for_problem(n, n, n, 1, batch=batch)
    c = c0.clone()
    bag.sgemm_batched(a, b, c, beta=1.0, depth=1, workspace=ws)
    torch.cuda.synchronize()
    assert bag.last_leaf_path() == "3xtf32"
    exact = c0.double() + a.double() @ b.double()
    assert float((c.double() - exact).norm() / exact.norm()) <= 2e-6
    assert bag.device_error() == 0


# The two prepared-operand leaf kernels: 256 x 256 tiles on a cluster of two
# SMs (tcgen05.mma.cta_group::2, the default) and 128 x 256 tiles on one SM
# (BAG_B200_PREP_KERNEL=single).  Same operands, same chunk folding:
# both within the FFMA bound, and close to each other.  Shapes cover ragged
# M/N (partial pair tiles), K tails that are not a multiple of the 32-k
# stage, fewer tiles than clusters, and batches.
@pytest.mark.parametrize("m,k,n,depth,batch", [
    (512, 2048, 768, 0, 1), (1032, 4096, 2056, 2, 1), (4096, 4096, 4096, 2, 1),
    (1000, 2048, 1160, 1, 2), (300, 1024, 104, 0, 3),
    (200, 1032, 136, 0, 1), (132, 1100, 260, 0, 2), (1536, 2064, 1032, 1, 1)])
def test_pair_and_single_leaf_kernels(tensor_mode, monkeypatch, m, k, n, depth, batch):
    import torch
    bag = tensor_mode
    g = torch.Generator(device="cuda").manual_seed(m * 3 + n + depth)
    a = torch.randn(batch, m, k, device="cuda", generator=g)
    b = torch.randn(batch, k, n, device="cuda", generator=g)
    ws = bag.Workspace.for_problem(n, m, k, depth, batch=batch)
    out = {}
    for kernel in ("tf32_pair", "tf32_single"):
        if kernel == "tf32_single":
            monkeypatch.setenv("BAG_B200_PREP_KERNEL", "single")
        c = torch.zeros(batch, m, n, device="cuda")
        bag.sgemm_batched(a, b, c, beta=0.0, depth=depth, workspace=ws)
        torch.cuda.synchronize()
        assert bag.last_leaf_kernel() == kernel
        assert bag.device_error() == 0
        out[kernel] = c
    monkeypatch.delenv("BAG_B200_PREP_KERNEL")
    exact = a.double() @ b.double()
    errs = {kk: float((c.double() - exact).norm() / exact.norm()) for kk, c in out.items()}
    bag.set_math_mode("ffma")
    ws_ffma = bag.Workspace.for_problem(n, m, k, depth, batch=batch)
    c_ff = torch.zeros(batch, m, n, device="cuda")
    bag.sgemm_batched(a, b, c_ff, beta=0.0, depth=depth, workspace=ws_ffma)
    torch.cuda.synchronize()
    bag.set_math_mode("3xtf32")
    ffma = float((c_ff.double() - exact).norm() / exact.norm())
    for kk, e in errs.items():
        assert e <= min(1.25 * ffma, 1e-4), (kk, e, ffma)
    diff = float((out["tf32_pair"] - out["tf32_single"]).double().norm() / exact.norm())
    assert diff <= 1e-6, diff


# Failure detection without a GPU fault: a wait on an mbarrier that nothing
# arrives on gives up after its limit, sets the device error word, and the
# context keeps working (the next product runs and is correct).
def test_bounded_wait_gives_up_and_context_survives(tensor_mode):
    import torch
    bag = tensor_mode
    assert bag.device_error() == 0
    assert bag.selftest_bounded_wait(2_000_000) is True
    assert bag.device_error() == 1
    assert bag.device_error() == 0   # read and cleared
    a, b = _operands(torch, 512, 2048, 512, seed=11)
    ws = bag.Workspace.for_problem(512, 512, 2048, 1)
    c, path = _sgemm(bag, torch, a, b, 1, "minimal", ws, "3xtf32")
    assert path == "3xtf32" and bag.last_leaf_kernel() == "tf32_pair"
    assert _rel(torch, c, a, b) <= 2e-6
    assert bag.device_error() == 0
    with pytest.raises(ValueError):   # BAG_ERR_INVALID
        bag.selftest_bounded_wait(0)


# Deferred inverse transform (one leaf shape): products store into their own
# buffers and one pass adds them into C -- accumulating (beta 1) or
# overwriting without zeroing C first (beta 0, C starts as garbage here).  At
# depth 1 (4 target blocks) a CTA slice is 512 or 1024 rows; the shapes below
# give a block shorter than one slice (500 rows), a last slice of 8 rows
# (520) and whole 1024-row slices.
@pytest.mark.parametrize("m,n,depth,beta", [
    (2048, 2048, 2, 0.0), (2048, 2048, 2, 1.0), (2064, 1040, 2, 1.0), (1040, 2064, 2, 0.0),
    (2048, 2048, 1, 0.0), (2048, 2048, 1, 1.0), (2000, 1000, 1, 0.0), (2064, 1040, 1, 1.0),
    (1040, 2064, 1, 0.0)])
def test_deferred_decode(tensor_mode, m, n, depth, beta):
    import torch
    bag = tensor_mode
    k = 2048 * depth
    assert bag.plan_dump(n, m, k, n, k, n, depth=depth)["decode"]["deferred"]
    g = torch.Generator(device="cuda").manual_seed(17)
    a = torch.randn(m, k, device="cuda", generator=g)
    b = torch.randn(k, n, device="cuda", generator=g)
    c0 = torch.randn(m, n, device="cuda", generator=g) if beta else torch.full((m, n), float("nan"), device="cuda")
    ws = bag.Workspace.for_problem(n, m, k, depth)
    c = c0.clone()
    bag.sgemm(a, b, c, beta=beta, depth=depth, workspace=ws)
    torch.cuda.synchronize()
    assert bag.last_leaf_kernel() == "tf32_pair" and bag.device_error() == 0
    exact = a.double() @ b.double() + (c0.double() if beta else 0.0)
    assert float((c.double() - exact).norm() / exact.norm()) <= 2e-6
    # Deterministic: the pass adds the products in plan order.
    c2 = c0.clone()
    bag.sgemm(a, b, c2, beta=beta, depth=depth, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(c, c2)


# Depth 3 on the prepared path: 343 products over several leaf launches and
# prepare-group launches (the decode stays fused: more products than the
# deferred pass takes).
def test_prepared_depth3(tensor_mode):
    import torch
    bag = tensor_mode
    n = 8192
    dump = bag.plan_dump(n, n, n, n, n, n, depth=3)
    assert len(dump["prepared"]) > 0 and not dump["decode"]["deferred"]
    a, b = _operands(torch, n, n, n, seed=33)
    ws = bag.Workspace.for_problem(n, n, n, 3)
    c, path = _sgemm(bag, torch, a, b, 3, "minimal", ws, "3xtf32")
    assert path == "3xtf32" and bag.last_leaf_kernel() == "tf32_pair" and bag.device_error() == 0
    exact = a.double() @ b.double()
    err = float((c.double() - exact).norm() / exact.norm())
    bag.set_math_mode("ffma")
    ws_f = bag.Workspace.for_problem(n, n, n, 3)
    c_f, _ = _sgemm(bag, torch, a, b, 3, "minimal", ws_f, "ffma")
    bag.set_math_mode("3xtf32")
    ffma = float((c_f.double() - exact).norm() / exact.norm())
    assert err <= min(1.25 * ffma, 1e-4), (err, ffma)


# Phase events: a prepared depth-2 call splits into stages | prepare | leaves |
# decode, each bracketed on the call's stream in that order.
def test_phase_events_split_a_prepared_call(tensor_mode):
    import torch
    bag = tensor_mode
    m = n = 2048
    k = 4096
    a, b = _operands(torch, m, k, n, seed=41)
    c = torch.zeros(m, n, device="cuda")
    ws = bag.Workspace.for_problem(n, m, k, 2)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    for e in ev:
        e.record()
    torch.cuda.synchronize()
    bag.profile_events(ev[2], ev[3])
    bag.profile_phase_events(ev[1], ev[4])
    try:
        ev[0].record()
        bag.sgemm(a, b, c, beta=0.0, depth=2, workspace=ws)
    finally:
        bag.profile_events(None, None)
        bag.profile_phase_events(None, None)
    torch.cuda.synchronize()
    spans = [ev[i].elapsed_time(ev[i + 1]) for i in range(4)]
    assert all(t >= 0 for t in spans), spans
    assert spans[2] > 0 and spans[3] > 0     # leaves, then the deferred decode
    with pytest.raises((ValueError, bag.BagError)):
        bag.profile_phase_events(ev[1], None)


def test_fused_fallback_warns_and_prepared_path_does_not(bag, cuda):
    """A 3xTF32 call whose workspace was created in FFMA mode runs the fused
    kernel and says so; one created in 3xTF32 mode runs the pair kernel quietly."""
    import warnings

    import torch
    n, depth = 2048, 1
    g = torch.Generator(device="cuda").manual_seed(17)
    a = torch.randn(n, n, device="cuda", generator=g)
    b = torch.randn(n, n, device="cuda", generator=g)
    c = torch.empty(n, n, device="cuda")
    ws_ffma = bag.Workspace.for_problem(n, n, n, depth)    # FFMA mode: no prepared region
    bag.set_math_mode("3xtf32")
    try:
        with pytest.warns(RuntimeWarning, match="fused-transform"):
            bag.sgemm(a, b, c, beta=0.0, depth=depth, workspace=ws_ffma)
        assert bag.last_leaf_kernel() == "tf32_fused"
        ws = bag.Workspace.for_problem(n, n, n, depth)
        with warnings.catch_warnings():
            warnings.simplefilter("error")
            bag.sgemm(a, b, c, beta=0.0, depth=depth, workspace=ws)
        assert bag.last_leaf_kernel() == "tf32_pair"
        torch.cuda.synchronize()
    finally:
        bag.set_math_mode("ffma")
    assert bag.device_error() == 0
