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
