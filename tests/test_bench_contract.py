"""bench.py pieces that need no GPU: every committed DRAM-traffic summary the
roofline cites parses, and the kernel names it reports have one."""

from __future__ import annotations

import glob
import os

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_every_traffic_summary_parses():
    files = sorted(glob.glob(os.path.join(ROOT, "profiles", "*traffic*.txt")))
    assert files
    for path in files:
        value = bench.read_traffic(os.path.basename(path))
        assert value is not None and value > 1e9, path


def test_roofline_kernels_have_traffic_summaries():
    for name in ("leaf_pair_cfg3_traffic.txt", "leaf_prep_cfg3_traffic.txt",
                 "leaf_tc_cfg3_traffic.txt", "leaf_gemm_cfg3_traffic.txt"):
        assert bench.read_traffic(name) is not None, name


def test_missing_or_malformed_summary_reads_as_none(tmp_path, monkeypatch):
    assert bench.read_traffic("no_such_file.txt") is None
    (tmp_path / "profiles").mkdir()
    (tmp_path / "profiles" / "bad.txt").write_text("traffic_bytes_per_full_launch: n/a\n")
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    assert bench.read_traffic("bad.txt") is None


def _sample(sm, power_cap=False, thermal=False):
    state = lambda on: "Active" if on else "Not Active"  # noqa: E731
    return (f"0, {sm}, 1965, 900.0, 0x0, {state(False)}, {state(thermal)}, "
            f"{state(False)}, {state(power_cap)}")


def test_clock_summary_keeps_the_timed_window():
    """The bench line's clocks: median SM clock and the throttle reasons of the
    samples inside the timed region only; outside samples are ignored."""
    s = bench.ClockSampler(0)
    s.lines = [(0.5, _sample(600, thermal=True)),          # before the region
               (1.1, _sample(1950)), (1.2, _sample(1965, power_cap=True)),
               (1.3, _sample(1900)),
               (9.0, _sample(300, thermal=True))]          # after it
    s.window = (1.0, 2.0)
    out = s.summary()
    assert out["sm_mhz"] == 1950 and out["sm_max_mhz"] == 1965
    assert out["reasons"] == ["sw_power_cap"]
    assert out["samples_in_timed_region"] == 3


def test_clock_summary_short_region_uses_nearest_samples_and_skips_bad_lines():
    s = bench.ClockSampler(0)
    s.lines = [(1.0, "garbage"), (1.04, _sample(1800, thermal=True)),
               (1.09, _sample(1900)), (5.0, _sample(100))]
    s.window = (1.05, 1.06)            # shorter than the 50 ms sampling period
    out = s.summary()
    assert out["samples_in_timed_region"] == 0
    assert out["sm_mhz"] == 1850 and "hw_thermal_slowdown" in out["reasons"]
    empty = bench.ClockSampler(0)
    assert empty.summary()["sm_mhz"] is None


def test_bench_configs_match_baseline():
    """Each --config reproduces the shape, seed, distribution and recursion
    depth that BASELINE.json states for it."""
    import json
    import re
    with open(os.path.join(ROOT, "BASELINE.json")) as f:
        text = json.load(f)["configs"]
    C = bench.CONFIGS
    expect = {   # config -> (index in BASELINE.json configs, M, N, K, batch, seed)
        "cfg1": (0, 512, 512, 512, 1, 0), "cfg2": (1, 4096, 4096, 4096, 1, 1),
        "cfg3": (2, 16384, 16384, 16384, 1, 2), "cfg4a": (3, 8192, 4096, 16384, 1, 3),
        "cfg4b": (3, 10000, 10000, 10000, 1, 3), "cfg5": (4, 2048, 2048, 2048, 64, 4),
    }
    for name, (idx, m, n, k, batch, seed) in expect.items():
        cfg, desc = C[name], text[idx]
        assert (cfg["m"], cfg["n"], cfg["k"], cfg["batch"], cfg["seed"]) == (m, n, k, batch, seed)
        assert re.search(rf"seed {seed}\b", desc), (name, desc)
        for size in {m, n, k}:
            assert str(size) in desc, (name, size)
        uniform = "uniform" in desc
        assert (cfg["dist"][0] == "uniform") == uniform
        if uniform:
            lo, hi = cfg["dist"][1:]
            assert f"[{lo:g},{hi:g})" in desc.replace(".0", "").replace(" ", "")
    assert "2 levels" in text[2] and C["cfg3"]["depth"] == 2
    assert "2 recursion levels" in text[1] and C["cfg2"]["depth"] in (1, 2)
    assert all(C[c]["depth"] == 1 for c in ("cfg1", "cfg4a", "cfg4b", "cfg5"))
