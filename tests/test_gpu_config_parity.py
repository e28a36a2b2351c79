"""Per-config parity on BASELINE's exact seeded inputs, against the reference's
own CUDA BAG.

Every BASELINE config draws A then B from ``numpy.random.default_rng(seed)``
exactly as ``bench.make_inputs`` does (row-major FP32).  The reference's
``bag_cuda::matmul`` (``include/bag/cuda/bag.cuh:249-260``, ColumnTile8 backend,
Batched schedule, Minimal basis; compiled unmodified from its headers into
``oracle/_ref/libbagref.so``) runs three times on the same inputs -- its
atomic epilogue makes the last bits vary -- and the median of its relative
Frobenius errors against an FP64 GEMM is the bound's base.  This library's
3xTF32 and FFMA paths must both stay within

    rel-F(mine) <= 1.25 x median rel-F(reference) and rel-F(mine) <= 1e-4

at equal recursion depth.  The reference is
column-major and square only:

* a row-major ``C = A B`` is its column-major ``C^T = B^T A^T``, so it is
  called with the pointers of B and A swapped; C starts at zero because the
  reference accumulates;
* cfg4a (8192 x 16384 x 4096) is composed from eight square 4096^3 calls on
  packed sub-blocks, accumulating into the two 4096-row blocks of C
  (C_i = sum_j A_ij B_j);
* cfg5 (64 problems of 2048^3) is 64 calls on one workspace, one stream.

cfg1 is also pinned to the reference's Triton ``bag_matmul``
(``src/bag_triton/bag.py:955``) run under ``TRITON_INTERPRET=1`` on cfg1's
exact inputs (``tests/golden/cfg1_triton_bag_n512.npz``, written by
``tests/golden/make_golden.py``).  Run with ``-s`` for one CONFIG_PARITY line
per case.
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN_CFG1 = os.path.join(ROOT, "tests", "golden", "cfg1_triton_bag_n512.npz")


@pytest.fixture(scope="module")
def ref():
    from bench import reference_cuda
    lib = reference_cuda()
    if lib is None:
        pytest.fail("oracle/_ref/libbagref.so is missing (build it with oracle/build_ref.py)")
    return lib


@pytest.fixture(scope="module")
def torch_mod(cuda):
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return torch


def _inputs(name):
    from bench import CONFIGS, make_inputs
    cfg = dict(CONFIGS[name])
    a, b = make_inputs(cfg)
    return cfg, a, b


def _rel_errors(torch, a, b, outs):
    """Relative Frobenius errors of each C in `outs` against an FP64 GEMM (GPU)."""
    from bench import frobenius_sums
    num, den = frobenius_sums(a, b, outs)
    return [(x / den) ** 0.5 for x in num]


def _reference_outputs(ref, torch, a, b, depth, runs=3):
    """`runs` fresh reference results C = A B (C starts at zero; the reference
    accumulates), through bench.reference_step: a batch is a loop of calls,
    cfg4a is composed from square 4096^3 calls on packed sub-blocks."""
    from bench import reference_step
    outs = []
    for _ in range(runs):
        c = torch.zeros(a.shape[:-1] + (b.shape[-1],), device="cuda")
        reference_step(ref, a, b, c, depth, "minimal", torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        outs.append(c)
    return outs


def _mine(bag, torch, a, b, depth, math):
    """C = A B through this library's public API in `math` mode; (C, leaf path)."""
    bag.set_math_mode(math)
    try:
        if a.ndim == 3:
            batch, m, k = a.shape
            n = b.shape[2]
            ws = bag.Workspace.for_problem(n, m, k, depth, batch=batch)
            c = torch.full((batch, m, n), float("nan"), device="cuda")
            bag.sgemm_batched(a, b, c, beta=0.0, depth=depth, workspace=ws)
        else:
            m, k = a.shape
            n = b.shape[1]
            ws = bag.Workspace.for_problem(n, m, k, depth)
            c = torch.full((m, n), float("nan"), device="cuda")
            bag.sgemm(a, b, c, beta=0.0, depth=depth, workspace=ws)
        torch.cuda.synchronize()
        path = bag.last_leaf_path()
        del ws
    finally:
        bag.set_math_mode("ffma")
    return c, path


# (config, depth): BASELINE's configs at the depths it names, cfg4b also at 2.
CASES = [("cfg1", 1), ("cfg2", 1), ("cfg2", 2), ("cfg3", 2), ("cfg4a", 1), ("cfg4b", 1),
         ("cfg4b", 2), ("cfg5", 1)]


@pytest.mark.parametrize("name,depth", CASES, ids=[f"{c}-d{d}" for c, d in CASES])
def test_config_within_reference_bound(bag, torch_mod, ref, name, depth):
    torch = torch_mod
    cfg, a_np, b_np = _inputs(name)
    a = torch.from_numpy(a_np).cuda()
    b = torch.from_numpy(b_np).cuda()
    del a_np, b_np
    refs = _reference_outputs(ref, torch, a, b, depth)
    ref_errs = _rel_errors(torch, a, b, refs)
    del refs
    torch.cuda.empty_cache()
    ref_err = float(np.median(ref_errs))
    line = {"config": name, "depth": depth, "reference_rel_f_runs": ref_errs,
            "reference_rel_f_median": ref_err}
    for math in ("3xtf32", "ffma"):
        c, path = _mine(bag, torch, a, b, depth, math)
        err = _rel_errors(torch, a, b, [c])[0]
        del c
        torch.cuda.empty_cache()
        line[f"{math}_rel_f"] = err
        line[f"{math}_leaf_path"] = path
        line[f"{math}_ratio"] = err / ref_err
    print("CONFIG_PARITY " + json.dumps(line), flush=True)
    assert bag.device_error() == 0
    for math in ("3xtf32", "ffma"):
        assert line[f"{math}_rel_f"] <= 1e-4, line
        assert line[f"{math}_rel_f"] <= 1.25 * ref_err, line


def test_cfg1_against_reference_triton_golden(bag, torch_mod):
    """cfg1's exact inputs through the reference's Triton bag_matmul (interpreter)."""
    torch = torch_mod
    z = np.load(GOLDEN_CFG1)
    cfg, a_np, b_np = _inputs("cfg1")
    assert np.array_equal(z["a_head"], a_np.ravel()[:64])   # same generator, same draws
    assert np.array_equal(z["b_head"], b_np.ravel()[:64])
    a, b = torch.from_numpy(a_np).cuda(), torch.from_numpy(b_np).cuda()
    exact = a_np.astype(np.float64) @ b_np.astype(np.float64)
    triton_err = float(np.linalg.norm(z["out"] - exact) / np.linalg.norm(exact))
    assert triton_err <= 3e-4                                # tests/triton/test_bag.py:60
    for math in ("3xtf32", "ffma"):
        c, _ = _mine(bag, torch, a, b, 1, math)
        got = c.cpu().numpy()
        err = float(np.linalg.norm(got - exact) / np.linalg.norm(exact))
        assert err <= 3e-4                                   # tests/triton/test_bag.py:60
        assert np.abs(got - exact).max() <= 2e-3 + 2e-5 * 512   # tests/triton/test_bag.py:61
        # Same algorithm: the results differ only by leaf summation order.
        assert float(np.linalg.norm(got - z["out"]) / np.linalg.norm(exact)) <= 2e-6
