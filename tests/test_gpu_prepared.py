"""The prepare pass of the 3xTF32 path, bit for bit.

After one call in 3xTF32 mode the workspace's prepared region holds every leaf
operand as TF32 hi rows then lo rows (k contiguous).  This test reads the
region back and compares it with a CPU restatement built from the plan dump
alone: each operand is its signed sum of mids, each mid its signed sum of
source blocks, evaluated in FP32 in order (the first term with its sign, then
one rounding per further term -- the reference's order, bag.cuh:69-73 and
124-135), then split hi = rn_tf32(x), lo = rn_tf32(x - hi) with round to
nearest, ties to even, on the 10-bit TF32 mantissa.  The comparison is exact:
the prepared operands must not change when the prepare pass is restructured,
and the kernels with compiled-in basis expressions must write the same bits
as the one that reads them from the plan.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from plan_sim import _view

pytestmark = pytest.mark.gpu


def _cudart():
    """The CUDA runtime the library loaded (for a device-to-host copy of raw memory)."""
    with open("/proc/self/maps") as f:
        for line in f:
            if "libcudart.so" in line:
                return ctypes.CDLL(line.split()[-1])
    pytest.fail("libcudart is not mapped into the process")


def _tf32_rne(x: np.ndarray) -> np.ndarray:
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x0FFF + ((u >> 13) & 1)) & 0xFFFFE000
    return u.astype(np.uint32).view(np.float32)


def _signed_sum(xs, signs):
    acc = None
    for x, sg in zip(xs, signs):
        x = (x * np.float32(sg)).astype(np.float32)
        acc = x if acc is None else (acc + x).astype(np.float32)
    return acc


CASES = [(256, 4096, 192, 2, "minimal"), (100, 4096, 72, 2, "minimal"),
         (128, 2048, 128, 1, "full"), (96, 4096, 64, 2, "winograd"), (64, 8192, 64, 3, "minimal"),
         (128, 4096, 96, 2, "classic"), (128, 2048, 64, 1, "classic"), (256, 4096, 256, 2, "full"),
         (64, 2048, 128, 1, "winograd"), (96, 2048, 96, 1, "minimal")]


@pytest.mark.parametrize("m,k,n,depth,basis", CASES)
def test_prepared_region_is_bit_exact(bag, cuda, m, k, n, depth, basis):
    import torch
    rng = np.random.default_rng(m + k + n + depth)
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((k, n), dtype=np.float32)
    # Column-major device copies: the plan dump describes the column-major call.
    ta = torch.from_numpy(np.ascontiguousarray(a.T)).cuda().t()
    tb = torch.from_numpy(np.ascontiguousarray(b.T)).cuda().t()
    tc = torch.zeros(n, m, device="cuda").t()
    bag.set_math_mode("3xtf32")
    try:
        plan = bag.plan_dump(m, n, k, m, k, m, depth, basis)
        ws = bag.Workspace.for_problem(m, n, k, depth, basis)
        bag.sgemm(ta, tb, tc, beta=0.0, depth=depth, basis=basis, workspace=ws)
        torch.cuda.synchronize()
        assert bag.last_leaf_kernel() in ("tf32_pair", "tf32_single")
        table = bag.last_prepare_table()
    finally:
        bag.set_math_mode("ffma")
    assert plan["prepared"] and plan["prepared_region"][0] == 3
    row_len = plan["prepared_row_len"]
    nrows = max(op["hi_row"] + 2 * op["rows"] for op in plan["prepared"])
    off = plan["prepared_region"][1]
    # The whole workspace: at depth >= 3 mids read blocks rounded there first.
    wsbuf = np.empty(plan["workspace_elements"], np.float32)
    st = _cudart().cudaMemcpy(ctypes.c_void_p(wsbuf.ctypes.data),
                              ctypes.c_void_p(bag.lib().bag_workspace_data(ws.handle)),
                              ctypes.c_size_t(wsbuf.nbytes), 2)
    assert st == 0
    region = wsbuf[off:off + nrows * row_len].reshape(nrows, row_len)
    bufs = [np.asfortranarray(a).ravel(order="F"), np.asfortranarray(b).ravel(order="F"), None,
            wsbuf]
    bad = []
    for j, op in enumerate(plan["prepared"]):
        shape = (op["rows"], op["cols"]) if op["transpose"] else (op["cols"], op["rows"])
        mids = [_signed_sum([_view(bufs[r[0]], r, *shape) for r, _ in mt], [c for _, c in mt])
                for mt, _ in op["terms"]]
        val = _signed_sum(mids, [c for _, c in op["terms"]])
        rows_k = val if op["transpose"] else val.T               # rows x k
        hi = _tf32_rne(rows_k)
        lo = _tf32_rne((rows_k - hi).astype(np.float32))
        got_hi = region[op["hi_row"]:op["hi_row"] + op["rows"]]
        got_lo = region[op["hi_row"] + op["rows"]:op["hi_row"] + 2 * op["rows"]]
        ok = (np.array_equal(got_hi[:, :op["cols"]].view(np.uint32), hi.view(np.uint32))
              and np.array_equal(got_lo[:, :op["cols"]].view(np.uint32), lo.view(np.uint32))
              and not got_hi[:, op["cols"]:].any() and not got_lo[:, op["cols"]:].any())
        if not ok:
            bad.append(j)
    assert not bad, f"{len(bad)} of {len(plan['prepared'])} prepared operands differ, e.g. {bad[:5]}"
    # Depths 1 and 2 of every basis run the kernel with the basis's operand
    # expressions compiled in; the region above is the same bit for bit.
    if depth <= 2:
        assert table == {"minimal": 1, "full": 2, "classic": 3, "winograd": 4}[basis], table
    exact = a.astype(np.float64) @ b.astype(np.float64)
    got = tc.cpu().numpy()
    # The product on those operands: 3xTF32 at this depth is ~1.3e-6 (N(0,1)).
    assert float(np.linalg.norm(got - exact) / np.linalg.norm(exact)) < 4e-6
    assert bag.device_error() == 0
