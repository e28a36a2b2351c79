"""Execute a dumped host plan (``bag_plan_dump``) in numpy -- test harness only.

This checks the C++ plan builder on CPU: every materialisation job and every
leaf product of the plan is evaluated in FP32 with numpy, in plan order, on
column-major buffers laid out exactly as the kernels would address them.
Plans of the prepared (3xTF32) path also carry the tree groups of the prepare
pass and, at depth >= 2, the deferred decode; both are executed as the kernels
order them (prep_tree_kernel: each mid's blocks, then each operand's mids, in
their own order, the first term with its sign; decode_kernel: per target, old
value plus the products in plan order).  Their deepest rounded operands are
virtual (never written by the library): the simulator writes them into a
fifth buffer from their definitions, like a materialisation job, so every
leaf operand is evaluated twice -- from its terms and by the tree groups -- and
the two must agree bit for bit.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
C_BUF, WS_BUF, VIRT_BUF = 2, 3, 4


def _view(buf: np.ndarray, ref, rows: int, cols: int) -> np.ndarray:
    _, off, ld = ref
    if rows == 0 or cols == 0:
        return np.zeros((rows, cols), F32)
    span = off + (cols - 1) * ld + rows
    assert span <= buf.size, f"plan reference {ref} {rows}x{cols} overruns a buffer of {buf.size}"
    return np.lib.stride_tricks.as_strided(buf[off:], shape=(rows, cols),
                                           strides=(buf.itemsize, buf.itemsize * ld))


def _signed_sum(xs, signs):
    acc = None
    for x, s in zip(xs, signs):
        x = (x.astype(F32) * F32(s)).astype(F32)
        acc = x if acc is None else (acc + x).astype(F32)
    return acc


def check_prep_groups(plan: dict) -> None:
    """Structural rules of the tree groups: every prepared operand sits in
    exactly one segment of a group of its own shape; a group has at most 16
    source blocks and 8 segments, a segment at most 4 mids and 8 operands;
    each operand's codes name its mids in order and each mid's codes its
    blocks in order; the operands' hi/lo row ranges of the prepared region do
    not overlap."""
    prepared, groups = plan["prepared"], plan["prep_groups"]
    seen = []
    for g in groups:
        assert 1 <= len(g["in"]) <= 16 and 1 <= len(g["segs"]) <= 8
        assert all(r[0] in (0, 1, 2, WS_BUF) for r in g["in"]), "a group reads a virtual block"
        for sg in g["segs"]:
            assert 1 <= len(sg["mids"]) <= 4 and 1 <= len(sg["ops"]) <= 8
            assert len(sg["expr"]) == len(sg["ops"])
            for j, codes in zip(sg["ops"], sg["expr"]):
                op = prepared[j]
                assert (op["rows"], op["cols"], op["transpose"]) == (g["rows"], g["cols"],
                                                                     g["transpose"])
                assert len(codes) == len(op["terms"])
                for code, (mid_terms, coef) in zip(codes, op["terms"]):
                    assert (1 if code > 0 else -1) == coef
                    mid = sg["mids"][abs(code) - 1]
                    assert len(mid) == len(mid_terms)
                    for mc, (ref, c) in zip(mid, mid_terms):
                        assert g["in"][abs(mc) - 1] == ref and (1 if mc > 0 else -1) == c
                seen.append(j)
    assert sorted(seen) == list(range(len(prepared)))
    spans = sorted((op["hi_row"], op["hi_row"] + 2 * op["rows"]) for op in prepared)
    for (_, end), (begin, _) in zip(spans, spans[1:]):
        assert end <= begin, "prepared operands overlap in the prepared region"
    for op in prepared:
        assert op["cols"] <= plan["prepared_row_len"]


def _write_prepared(plan: dict, bufs) -> None:
    """Evaluate every tree group and store its operands in the prepared region
    of the workspace as the kernels lay it out: operand j occupies region rows
    [hi_row, hi_row + 2 * rows) (hi rows, then lo rows) of
    ``prepared_row_len`` k values each, zero past its k extent.  Here the hi
    rows hold the FP32 value and the lo rows zero (the TF32 split itself is
    the GPU tests' business).  All groups of a launch read their sources
    before any output lands, so every group is evaluated first."""
    values = {}
    for g in plan["prep_groups"]:
        # Natural (column-major) shape of the source blocks: a left operand
        # (transposed into k-contiguous rows) is rows x cols, a right one cols x rows.
        shape = (g["rows"], g["cols"]) if g["transpose"] else (g["cols"], g["rows"])
        ins = [_view(bufs[r[0]], r, *shape).copy() for r in g["in"]]
        for sg in g["segs"]:
            mids = [_signed_sum([ins[abs(c) - 1] for c in m], [1 if c > 0 else -1 for c in m])
                    for m in sg["mids"]]
            for j, codes in zip(sg["ops"], sg["expr"]):
                values[j] = _signed_sum([mids[abs(c) - 1] for c in codes],
                                        [1 if c > 0 else -1 for c in codes])
    region = _prepared_region(plan, bufs)
    for j, op in enumerate(plan["prepared"]):
        rows_k = values[j] if op["transpose"] else values[j].T   # rows x k
        hi = op["hi_row"]
        region[:, hi:hi + 2 * op["rows"]] = 0
        region[:op["cols"], hi:hi + op["rows"]] = rows_k.T


def _prepared_region(plan: dict, bufs) -> np.ndarray:
    ref = plan["prepared_region"]
    nrows = max(op["hi_row"] + 2 * op["rows"] for op in plan["prepared"])
    assert ref[0] == WS_BUF and ref[2] == plan["prepared_row_len"]
    return _view(bufs[WS_BUF], ref, plan["prepared_row_len"], nrows)


def _read_prepared(plan: dict, bufs, j: int) -> np.ndarray:
    """Operand j back from the region (hi + lo), rows x k."""
    op, region = plan["prepared"][j], _prepared_region(plan, bufs)
    hi, rows = op["hi_row"], op["rows"]
    assert not np.any(region[op["cols"]:, hi:hi + 2 * rows]), "prepared padding is not zero"
    return (region[:op["cols"], hi:hi + rows] + region[:op["cols"], hi + rows:hi + 2 * rows]).T


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

    virt = plan.get("virtual", [])
    vsize = max([v["out"][1] + (v["cols"] - 1) * v["out"][2] + v["rows"] for v in virt] + [1])
    bufs = [flat(a, m, k, lda), flat(b, k, n, ldb), flat(c, m, n, ldc),
            np.full(max(plan["workspace_elements"], 1), np.nan, F32),
            np.full(vsize, np.nan, F32)]
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
    # Virtual blocks: written here from their definitions (the library never
    # writes them; its prepare pass evaluates them inside the tree groups).
    for v in virt:
        assert v["out"][0] == VIRT_BUF
        rows, cols = v["rows"], v["cols"]
        terms = [(_view(bufs[r[0]], r, rows, cols), coef) for r, coef in v["terms"]]
        assert all(r[0] != VIRT_BUF for r, _ in v["terms"]), "virtual block of virtual blocks"
        _view(bufs[VIRT_BUF], v["out"], rows, cols)[...] = _signed_sum(
            [x for x, _ in terms], [cf for _, cf in terms])
    prepared = bool(plan.get("prepared"))
    assert prepared or not virt, "virtual blocks outside the prepared path"
    if prepared:
        check_prep_groups(plan)
        _write_prepared(plan, bufs)
    decode = plan.get("decode", {})
    deferred = bool(decode.get("deferred"))
    for leaf in plan["leaves"]:
        lm, ln, lk = leaf["m"], leaf["n"], leaf["k"]

        def operand(terms, rows, cols):
            return _signed_sum([_view(bufs[ref[0]], ref, rows, cols) for ref, _ in terms],
                               [coef for _, coef in terms])

        left = operand(leaf["left"], lm, lk)
        right = operand(leaf["right"], lk, ln)
        assert np.all(np.isfinite(left)) and np.all(np.isfinite(right)), "read of unwritten workspace"
        if prepared:
            # The leaf multiplies its prepared operands, read back from the
            # region after every earlier leaf's stores: they must equal the
            # operand sums bit for bit.
            assert np.array_equal(_read_prepared(plan, bufs, leaf["prep_l"]), left)
            assert np.array_equal(_read_prepared(plan, bufs, leaf["prep_r"]).T, right)
        prod = (left.astype(F32) @ right.astype(F32)).astype(F32)
        for ref, coef in leaf["out"]:
            v = _view(bufs[ref[0]], ref, lm, ln)
            if ref[0] == WS_BUF:
                assert deferred and ref in decode["buffers"], "workspace output without a decode"
                v[...] = (F32(coef) * prod).astype(F32)
            else:
                assert ref[0] == C_BUF, "outputs must target C or a decode buffer"
                v[...] = (v + F32(coef) * prod).astype(F32)
    if deferred:
        dm, dn = decode["m"], decode["n"]
        prods = [_view(bufs[WS_BUF], r, dm, dn).copy() for r in decode["buffers"]]
        for t, tref in enumerate(decode["target_refs"]):
            assert tref[0] == C_BUF
            v = _view(bufs[C_BUF], tref, dm, dn)
            acc = v.copy()
            for p, terms in enumerate(decode["terms"]):
                for tt, coef in terms:
                    if tt == t:
                        acc = (acc + F32(coef) * prods[p]).astype(F32)
            v[...] = acc
    return _view(bufs[C_BUF], (C_BUF, 0, ldc), m, n).copy()
