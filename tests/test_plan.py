"""CPU tests of the host plan builder (no GPU): the dumped plan, executed in
numpy by ``tests/plan_sim.py``, must compute C + A@B for every basis, depth
and ragged or rectangular shape, and must round transformed operands where
the reference does."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import bag_oracle as O
from plan_sim import run_plan

CASES = [
    # m, k, n, depth, basis
    (64, 64, 64, 1, "minimal"),
    (64, 64, 64, 2, "minimal"),
    (64, 64, 64, 3, "minimal"),
    (64, 64, 64, 1, "full"),
    (64, 64, 64, 2, "full"),
    (64, 64, 64, 1, "classic"),
    (64, 64, 64, 2, "classic"),
    (72, 40, 56, 1, "minimal"),      # rectangular
    (77, 53, 61, 2, "minimal"),      # ragged: peeled strips
    (3, 5, 7, 1, "minimal"),         # smaller than one BAG block: plain GEMM
    (128, 256, 64, 2, "full"),
    (100, 100, 100, 1, "minimal"),   # 10000-style: halves to a non-multiple of 8
    (40, 0, 24, 1, "minimal"),       # empty K
    (48, 48, 48, 0, "minimal"),      # depth 0: plain GEMM
]


@pytest.mark.parametrize("m,k,n,depth,basis", CASES)
def test_plan_computes_gemm(bag, m, k, n, depth, basis):
    rng = np.random.default_rng(m * 7 + k * 3 + n + depth)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    c = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    lda, ldb, ldc = m + 4, k + 8, m
    plan = bag.plan_dump(m, n, k, lda, ldb, ldc, depth, basis)
    got = run_plan(plan, a, b, c, lda, ldb, ldc)
    assert O.rel_frobenius(got, O.fp64_matmul(a, b, c)) < 1e-6 * max(depth, 1) + 1e-7


@pytest.mark.parametrize("depth", [1, 2])
@pytest.mark.parametrize("basis", ["minimal", "full"])
def test_plan_operands_round_like_reference(bag, depth, basis):
    """Leaf products see bit-identical operands to the oracle's recursion.

    With exactly representable inputs (multiples of 2^-16) every product of
    two operands is exact in FP64, so comparing against the oracle run in the
    same association order isolates the operand rounding.
    """
    n = 32
    a = O.hash_matrix(n, n, 11)
    b = O.hash_matrix(n, n, 23)
    plan = bag.plan_dump(n, n, n, n, n, n, depth, basis)
    got = run_plan(plan, a, b, np.zeros((n, n), np.float32), n, n, n)
    ref = O.bag_product(a, b, depth, basis)
    assert O.rel_frobenius(got, ref) < 1e-6


def test_plan_shapes_and_counts(bag):
    p1 = bag.plan_dump(64, 64, 64, 64, 64, 64, 1, "minimal")
    assert len(p1["leaves"]) == 7 and p1["workspace_elements"] == 0 and p1["stages"] == []
    # Direct decode: 14 output updates per level (M1:2 M2:2 M3:3 M4:1 M5:4 M6:1 M7:1).
    assert sum(len(l["out"]) for l in p1["leaves"]) == 14
    # Fused operand terms per level: 14 left and 14 right (max 4: SA - A11, SB - B11).
    assert sum(len(l["left"]) for l in p1["leaves"]) == 14
    assert max(len(l["left"]) for l in p1["leaves"]) == 4
    p2 = bag.plan_dump(64, 64, 64, 64, 64, 64, 2, "minimal")
    assert len(p2["leaves"]) == 49
    assert sum(len(l["out"]) for l in p2["leaves"]) == 14 * 14
    # One pass per operand rounds the four multi-term outer operands.
    assert len(p2["stages"]) == 1 and len(p2["stages"][0]) == 2
    assert all(len(j["out"]) == 4 for j in p2["stages"][0])
    pf = bag.plan_dump(64, 64, 64, 64, 64, 64, 1, "full")
    assert len(pf["stages"]) == 1 and len(pf["stages"][0]) == 2
    assert max(len(l["left"]) for l in pf["leaves"]) == 2


def test_plan_peels_ragged_edges(bag):
    p = bag.plan_dump(77, 61, 53, 80, 56, 77, 2, "minimal")
    # 49 BAG leaves on the 64x48x64 core plus the K, M and N strips.
    assert len(p["leaves"]) == 52
    strips = p["leaves"][49:]
    assert [(s["m"], s["n"], s["k"]) for s in strips] == [(64, 48, 5), (13, 61, 53), (64, 13, 53)]


def test_plan_workspace_alignment(bag):
    p = bag.plan_dump(200, 200, 200, 200, 200, 200, 2, "full")
    for stage in p["stages"]:
        for job in stage:
            for ref in job["out"]:
                assert ref[0] == 3 and ref[1] % 64 == 0 and ref[2] % 4 == 0


@pytest.mark.parametrize("mode,n,leaf", [("3xtf32", 2048, 2048), ("3xtf32", 4096, 2048),
                                         ("3xtf32", 8192, 4096), ("3xtf32", 10000, 5000),
                                         ("3xtf32", 16384, 4096), ("3xtf32", 32768, 4096),
                                         ("ffma", 4096, 1024), ("ffma", 8192, 2048),
                                         ("ffma", 16384, 2048), ("ffma", 512, 512)])
def test_auto_depth_follows_the_measured_policy(built_lib, mode, n, leaf):
    import bag_b200 as bag
    bag.set_math_mode(mode)
    try:
        pl = bag.plan_dump(n, n, n, n, n, n, "auto", "minimal")
    finally:
        bag.set_math_mode("ffma")
    assert {l["m"] for l in pl["leaves"]} == {leaf}
    depth = round(n / leaf).bit_length() - 1
    assert len(pl["leaves"]) == 7 ** depth


def test_winograd_plan_has_the_15_addition_structure(built_lib):
    import bag_b200 as bag
    pl = bag.plan_dump(64, 64, 64, 64, 64, 64, 1, "winograd")
    leaves = pl["leaves"]
    assert len(leaves) == 7
    # Operand term counts (S/T intermediates flattened) and C updates per product.
    assert [(len(l["left"]), len(l["right"]), len(l["out"])) for l in leaves] == [
        (1, 1, 4), (1, 1, 1), (4, 1, 1), (1, 4, 1), (2, 2, 2), (3, 3, 3), (2, 2, 2)]
    assert len(bag.plan_dump(64, 64, 64, 64, 64, 64, 2, "winograd")["leaves"]) == 49


# Prepared (3xTF32) plans: leaves need K >= 1024, so these keep M and N small
# and K long.  (m, k, n, depth, basis, deferred decode expected)
PREPARED = [
    (64, 2048, 64, 1, "minimal", True),     # depth 1: 7 products, 4 targets: deferred decode
    (64, 2048, 64, 1, "classic", True),
    (64, 4096, 64, 2, "minimal", True),     # 49 products, 16 targets
    (64, 4096, 48, 2, "full", True),
    (64, 4096, 64, 2, "winograd", True),
    (64, 4096, 64, 2, "classic", True),
    (77, 4096, 61, 2, "minimal", False),    # peeled M/N strips: leaf shapes differ
    (32, 8192, 32, 3, "minimal", False),    # 343 products: above the decode's 64
]


@pytest.mark.parametrize("m,k,n,depth,basis,deferred", PREPARED)
def test_prepared_plan_computes_gemm(built_lib, m, k, n, depth, basis, deferred):
    """The prepared path's plan -- stages, prepare groups, leaf products on
    the prepared region and the deferred decode -- executed in numpy."""
    import bag_b200 as bag
    rng = np.random.default_rng(m + k + n + depth)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    c = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    bag.set_math_mode("3xtf32")
    try:
        plan = bag.plan_dump(m, n, k, m, k, m, depth, basis)
    finally:
        bag.set_math_mode("ffma")
    assert plan["prepared"] and plan["prep_groups"]
    assert plan["decode"]["deferred"] is deferred
    if deferred:
        assert all(r[0] == 3 and len(l["out"]) == 1 for l in plan["leaves"] for r, _ in l["out"])
        assert len(plan["decode"]["buffers"]) == len(plan["leaves"])
        assert len(plan["decode"]["target_refs"]) == 4 ** depth
    got = run_plan(plan, a, b, c, m, k, m)
    assert O.rel_frobenius(got, O.fp64_matmul(a, b, c)) < 5e-6 * depth


def test_prepare_groups_share_source_blocks(built_lib):
    """At depth 2 the 98 prepared operands (49 left, 49 right) fold into one
    tree group per side: the 16 sub-blocks of A's (B's) quadrants are read
    once per tile, each outer product is a segment whose 4 mids are the
    sub-blocks of its outer operand -- the operand the reference rounds
    before splitting (prepare_child), evaluated in the same order and never
    written to memory -- and its 7 inner operands are signed sums of those
    mids.  There are no materialisation stages, and the workspace holds only
    the prepared region and the deferred decode's product buffers."""
    import bag_b200 as bag
    bag.set_math_mode("3xtf32")
    try:
        plan = bag.plan_dump(64, 64, 4096, 64, 4096, 64, 2, "minimal")
    finally:
        bag.set_math_mode("ffma")
    ops, groups = plan["prepared"], plan["prep_groups"]
    assert len(ops) == 98 and plan["stages"] == []
    assert sum(len(op["terms"]) for op in ops) == 196
    assert len(groups) == 2 and sorted(g["transpose"] for g in groups) == [False, True]
    for g in groups:
        assert len(g["in"]) == 16 and len(g["segs"]) == 7
        assert all(len(sg["mids"]) == 4 and len(sg["ops"]) == 7 for sg in g["segs"])
    # The four multi-term outer operands per side (M1, M2, M3, M6 / M7) stay virtual.
    assert len(plan["virtual"]) == 8
    region_rows = sum(2 * op["rows"] for op in ops)
    decode = 49 * 32 * 32   # 49 product buffers of 32 x 32 (ld 32)
    assert plan["workspace_elements"] <= region_rows * plan["prepared_row_len"] + decode + 64 * 50


def test_ffma_plans_carry_no_prepared_operands(bag):
    plan = bag.plan_dump(64, 64, 4096, 64, 4096, 64, 2, "minimal")
    assert plan["prepared"] == [] and plan["prep_groups"] == []
    assert plan["prepared_region"] is None and not plan["decode"]["deferred"]


def test_plan_sim_catches_a_corrupted_prepared_plan(built_lib):
    """The checks above have teeth: a flipped sign in an operand's mids or in a
    mid's blocks, two segment outputs swapped, a wrong virtual block or a
    misrouted decode term is caught."""
    import copy

    import bag_b200 as bag
    m = n = 64
    k = 4096
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    c = np.zeros((m, n), np.float32)
    bag.set_math_mode("3xtf32")
    try:
        plan = bag.plan_dump(m, n, k, m, k, m, 2, "minimal")
    finally:
        bag.set_math_mode("ffma")
    ref = O.fp64_matmul(a, b, c)
    assert O.rel_frobenius(run_plan(plan, a, b, c, m, k, m), ref) < 1e-5

    bad = copy.deepcopy(plan)
    code = bad["prep_groups"][1]["segs"][3]["expr"][2]
    code[-1] = -code[-1]
    with pytest.raises(AssertionError):
        run_plan(bad, a, b, c, m, k, m)

    bad = copy.deepcopy(plan)
    mid = bad["prep_groups"][0]["segs"][2]["mids"][1]
    mid[-1] = -mid[-1]
    with pytest.raises(AssertionError):
        run_plan(bad, a, b, c, m, k, m)

    bad = copy.deepcopy(plan)
    sg = bad["prep_groups"][0]["segs"][0]
    sg["ops"][0], sg["ops"][1] = sg["ops"][1], sg["ops"][0]
    with pytest.raises(AssertionError):
        run_plan(bad, a, b, c, m, k, m)

    bad = copy.deepcopy(plan)
    term = bad["virtual"][2]["terms"][1]
    term[1] = -term[1]
    with pytest.raises(AssertionError):
        run_plan(bad, a, b, c, m, k, m)

    bad = copy.deepcopy(plan)
    term = bad["decode"]["terms"][10][0]
    term[0] = (term[0] + 1) % len(bad["decode"]["target_refs"])
    assert O.rel_frobenius(run_plan(bad, a, b, c, m, k, m), ref) > 1e-2


@pytest.mark.parametrize("m,k,n,depth,basis,table", [
    (2048, 2048, 2048, 1, "minimal", 1), (4096, 4096, 4096, 2, "minimal", 1),
    (2048, 2048, 2048, 1, "full", 2), (4096, 4096, 4096, 2, "full", 2),
    (2048, 2048, 2048, 1, "classic", 3), (4096, 4096, 4096, 2, "classic", 3),
    (2048, 2048, 2048, 1, "winograd", 4), (4096, 4096, 4096, 2, "winograd", 4),
    (64, 8192, 64, 3, "minimal", 1)])
def test_prepare_launch_takes_the_compiled_in_tables(built_lib, m, k, n, depth, basis, table):
    """The prepare kernel has each basis's operand expressions compiled in
    (bag_tc3_kernel.cu) and takes them only when every segment the plan
    builder produced matches; this pins the builder's expression order to
    those tables, so a change to either shows here instead of as a silent
    fall back to the plan-reading kernel."""
    import bag_b200 as bag
    bag.set_math_mode("3xtf32")
    try:
        plan = bag.plan_dump(m, n, k, m, k, m, depth, basis)
    finally:
        bag.set_math_mode("ffma")
    launches = plan["prepare_tables"]
    assert launches and all(l["basis_tables"] == table for l in launches)
    assert all(all(launch["groups"]) for launch in launches)


def test_ragged_prepare_keeps_the_tables_for_the_main_groups(built_lib):
    """Peeled strips of a ragged shape are single-input groups: they read
    their terms from the plan inside the same launch, the main groups keep
    the compiled-in tables."""
    import bag_b200 as bag
    bag.set_math_mode("3xtf32")
    try:
        plan = bag.plan_dump(100, 72, 4096, 100, 4096, 100, 2, "minimal")
    finally:
        bag.set_math_mode("ffma")
    (launch,) = plan["prepare_tables"]
    assert launch["basis_tables"] == 1
    groups = plan["prep_groups"]
    assert len(launch["groups"]) == len(groups)
    for flag, g in zip(launch["groups"], groups):
        assert flag == (1 if len(g["in"]) > 1 else 0)
