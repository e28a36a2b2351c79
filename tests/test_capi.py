"""CPU tests of the C ABI: the library loads, exports every declared symbol,
and its host-side validation matches the reference's rules and errors.
No kernel is launched here."""

from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "bag_capi.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bag_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for expected in ("bag_matmul", "bag_sgemm_ex", "bag_sgemm_batched", "bag_primitive",
                     "bag_strassen_one_level", "bag_workspace_create", "bag_last_error"):
        assert expected in names


def test_library_exports_every_declared_symbol(built_lib):
    out = subprocess.run(["nm", "-D", "--defined-only", built_lib], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (bag_[a-z0-9_]+)$", out, flags=re.M))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, f"declared but not exported: {missing}"


def test_python_signatures_cover_header(bag):
    assert set(bag.SIGNATURES) == set(declared_functions())
    for name in bag.SIGNATURES:
        assert getattr(bag.lib(), name) is not None


def test_version(bag):
    assert b"sm_100a" in bag.lib().bag_version()


@pytest.mark.parametrize("n,depth,basis,expected", [
    (16, 1, "minimal", 16 * 16 + 16 * 16 // 2),
    (16, 1, "full", 3 * 16 * 16),
    (64, 3, "minimal", 64 * 64 * 3 // 2),
])
def test_local_elements_matches_reference(bag, n, depth, basis, expected):
    # bag.cuh:23-30
    assert bag.local_elements(n, depth, basis) == expected


@pytest.mark.parametrize("n,depth", [(12, 1), (24, 2), (16, 0), (0, 1)])
def test_local_elements_rejects_like_reference(bag, n, depth):
    with pytest.raises(ValueError):
        bag.local_elements(n, depth)


@pytest.mark.parametrize("backend,s,valid", [
    ("huge", 128, True), ("huge", 192, False), ("large", 64, True), ("large", 96, False),
    ("medium", 96, True), ("column_tile64_k16_r4x8", 12, True), ("column_tile64_k16_r4x8", 6, False),
    ("legacy", 384, True), ("legacy", 400, False), ("legacy", 2048, True),
])
def test_valid_shape_matches_reference(bag, backend, s, valid):
    # strassen.cuh:57-66
    assert bag.valid_shape(backend, s) is valid


def test_errors_are_status_codes_not_exceptions(bag):
    lib = bag.lib()
    # Null workspace, bad backend, bad schedule: BAG_ERR_WORKSPACE / INVALID.
    assert lib.bag_matmul(None, None, None, 16, None, None, 37, 2) == 3
    assert b"workspace" in lib.bag_last_error()
    assert lib.bag_primitive(2, 0, 1, 0, 1, None, None, None, None, None, None, 4, 4, 4,
                             4, 4, 4, 4, 4, 4, None) == 1
    assert b"delta" in lib.bag_last_error()
    assert lib.bag_sgemm_ex(7, 4, 4, 4, None, 4, None, 4, None, 4, 1.0, 1, 0, None, None) == 1
    assert lib.bag_sgemm_ex(0, 4, 4, 4, None, 4, None, 4, None, 4, 0.5, 1, 0, None, None) == 4
    assert lib.bag_strassen_one_level(37, 6, None, None, None, 12, None) == 2
    # strassen.cuh:228-231: shape first, then "selected backend requires atomic updates".
    assert lib.bag_strassen_one_level(0, 1, None, None, None, 16, None) == 2
    assert lib.bag_strassen_one_level(0, 1, None, None, None, 64, None) == 4
    valid = ctypes.c_int()
    assert lib.bag_valid_shape(99, 16, ctypes.byref(valid)) == 1


def test_empty_problems_are_no_ops(bag):
    lib = bag.lib()
    # m == 0 or n == 0 returns before touching the device.
    assert lib.bag_sgemm_ex(0, 0, 8, 8, None, 1, None, 8, None, 1, 1.0, 1, 0, None, None) == 0
    assert lib.bag_primitive(0, 0, 1, 0, 1, None, None, None, None, None, None, 0, 4, 4,
                             1, 1, 4, 4, 1, 1, None) == 0


def test_plan_dump_without_gpu(bag):
    plan = bag.plan_dump(16, 16, 16, 16, 16, 16, 1, "minimal")
    assert len(plan["leaves"]) == 7


def test_workspace_sizes(bag):
    # Depth-1 Minimal fuses every transform: no workspace; deeper plans round
    # the outer operands into 8 quarter-size blocks (4 per operand).
    plan1 = bag.plan_dump(1024, 1024, 1024, 1024, 1024, 1024, 1, "minimal")
    plan2 = bag.plan_dump(1024, 1024, 1024, 1024, 1024, 1024, 2, "minimal")
    assert plan1["workspace_elements"] == 0
    assert plan2["workspace_elements"] == 8 * 512 * 512


def test_profiling_hooks_take_both_events_or_neither(bag):
    """The measurement hooks store caller-owned events per host thread; a
    half-set pair is refused (BAG_ERR_INVALID) and NULL, NULL turns a pair off.
    Any non-null handle works as a token here: nothing is recorded without a
    call on a GPU."""
    lib = bag.lib()
    token = ctypes.c_void_p(0x1000)
    assert lib.bag_profile_set_events(token, None) == 1
    assert b"both" in lib.bag_last_error()
    assert lib.bag_profile_set_phase_events(None, token) == 1
    assert b"both" in lib.bag_last_error()
    assert lib.bag_profile_set_events(None, None) == 0
    assert lib.bag_profile_set_phase_events(None, None) == 0
    # Counting launches needs no device either.
    assert lib.bag_launch_count() >= 0


def test_workspace_bytes_for_follows_the_math_mode():
    """bag_workspace_bytes_for sizes a workspace as bag_workspace_create_ex would
    on a thread in that mode: in 3XTF32 the prepared operands (and the deferred
    decode's product buffers) come on top of the FFMA plan's rounded operands."""
    import bag_b200 as bag
    n, depth = 16384, 2
    ffma = bag.workspace_bytes_for(n, n, n, depth, math="ffma")
    tf32 = bag.workspace_bytes_for(n, n, n, depth, math="3xtf32")
    assert ffma == 8 * (n // 2) ** 2 * 4                         # 8 outer operands of 8192^2
    assert tf32 > ffma + 98 * 2 * 4096 * 4096 * 4                # + 98 operands, hi and lo planes
    previous = bag.get_math_mode()
    try:
        for mode, want in (("ffma", ffma), ("3xtf32", tf32)):
            bag.set_math_mode(mode)
            assert bag.plan_dump(n, n, n, n, n, n, depth)["workspace_elements"] * 4 == want
            assert bag.workspace_bytes_for(n, n, n, depth) == want   # this thread's mode
    finally:
        bag.set_math_mode(previous)
    # Leaves shorter than 1024 stay on FFMA: no prepared region.
    assert bag.workspace_bytes_for(1024, 1024, 1024, 1, math="3xtf32") == \
        bag.workspace_bytes_for(1024, 1024, 1024, 1, math="ffma")
    assert bag.workspace_bytes_for(512, 512, 512, 3, batch=4, math="ffma") == \
        4 * bag.workspace_bytes_for(512, 512, 512, 3, math="ffma")
    with pytest.raises(ValueError):
        bag.workspace_bytes_for(-1, 8, 8, 1)


def test_device_allocation_counter_without_a_gpu():
    import bag_b200 as bag
    before = bag.device_allocations()
    bag.workspace_bytes_for(4096, 4096, 4096, 2, math="3xtf32")
    bag.plan_dump(256, 256, 256, 256, 256, 256, 2)
    assert bag.device_allocations() == before   # sizing and planning allocate nothing


@pytest.mark.parametrize("value,want,warns", [(None, "ffma", False), ("ffma", "ffma", False),
                                              ("3xtf32", "3xtf32", False),
                                              ("tf32", "ffma", True)])
def test_math_mode_default_from_environment(value, want, warns):
    """BAG_B200_MATH sets the mode every host thread starts in (the main thread
    and a new one alike); an unknown value keeps FFMA and says so on stderr."""
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = {k: v for k, v in os.environ.items() if k != "BAG_B200_MATH"}
    if value is not None:
        env["BAG_B200_MATH"] = value
    prog = ("import threading, bag_b200 as bag\n"
            "seen = []\n"
            "t = threading.Thread(target=lambda: seen.append(bag.get_math_mode()))\n"
            "t.start(); t.join()\n"
            "print(bag.get_math_mode(), seen[0])\n")
    r = subprocess.run([sys.executable, "-c", prog], cwd=root, env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.split() == [want, want]
    assert ("BAG_B200_MATH" in r.stderr) == warns
