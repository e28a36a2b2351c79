"""Execute a dumped host plan (``bag_plan_dump``) in numpy -- test harness only.

This checks the C++ plan builder on CPU: every materialisation job and every
leaf product of the plan is evaluated in FP32 with numpy, in plan order, on
column-major buffers laid out exactly as the kernels would address them.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def _view(buf: np.ndarray, ref, rows: int, cols: int) -> np.ndarray:
    _, off, ld = ref
    if rows == 0 or cols == 0:
        return np.zeros((rows, cols), F32)
    span = off + (cols - 1) * ld + rows
    assert span <= buf.size, f"plan reference {ref} {rows}x{cols} overruns a buffer of {buf.size}"
    return np.lib.stride_tricks.as_strided(buf[off:], shape=(rows, cols),
                                           strides=(buf.itemsize, buf.itemsize * ld))


def run_plan(plan: dict, a: np.ndarray, b: np.ndarray, c: np.ndarray,
             lda: int, ldb: int, ldc: int) -> np.ndarray:
    """Apply ``plan`` to column-major a (m x k), b (k x n), c (m x n); returns new C."""
    m, k = a.shape
    n = b.shape[1]

    def flat(x, rows, cols, ld):
        buf = np.zeros(max(ld * max(cols, 1), 1), F32)
        if rows and cols:
            _view(buf, (0, 0, ld), rows, cols)[...] = x
        return buf

    bufs = [flat(a, m, k, lda), flat(b, k, n, ldb), flat(c, m, n, ldc),
            np.full(max(plan["workspace_elements"], 1), np.nan, F32)]
    for stage in plan["stages"]:
        for job in stage:
            rows, cols = job["rows"], job["cols"]
            ins = [_view(bufs[r[0]], r, rows, cols).copy() for r in job["in"]]
            for out_ref, expr in zip(job["out"], job["expr"]):
                acc = None
                for code in expr:
                    x = ins[abs(code) - 1] * F32(1 if code > 0 else -1)
                    acc = x.astype(F32) if acc is None else (acc + x).astype(F32)
                _view(bufs[out_ref[0]], out_ref, rows, cols)[...] = acc
    for leaf in plan["leaves"]:
        lm, ln, lk = leaf["m"], leaf["n"], leaf["k"]

        def operand(terms, rows, cols):
            acc = None
            for ref, coef in terms:
                x = _view(bufs[ref[0]], ref, rows, cols).astype(F32) * F32(coef)
                acc = x if acc is None else (acc + x).astype(F32)
            return acc

        left = operand(leaf["left"], lm, lk)
        right = operand(leaf["right"], lk, ln)
        assert np.all(np.isfinite(left)) and np.all(np.isfinite(right)), "read of unwritten workspace"
        prod = (left.astype(F32) @ right.astype(F32)).astype(F32)
        for ref, coef in leaf["out"]:
            assert ref[0] == 2, "outputs must target C"
            v = _view(bufs[2], ref, lm, ln)
            v[...] = (v + F32(coef) * prod).astype(F32)
    return _view(bufs[2], (2, 0, ldc), m, n).copy()
