"""The reference-format benchmark driver (bag_b200/benchmark.py).

CPU: its input generator against the restated reference hash
(fp32_baseline.cu:26-32) and its sample positions against std::mt19937 as the
reference draws them (fp32_baseline.cu:126-131).  GPU: a small run in each
math mode writes the four files with the reference's headers and passes the
reference's FP64 limits."""

from __future__ import annotations

import csv
import json
import os
import shutil
import subprocess

import numpy as np
import pytest

from bag_b200 import benchmark as D
from oracle import bag_oracle as O


def test_hash_values_match_the_reference_generator():
    import torch
    idx = np.concatenate([np.arange(0, 5000), np.array([2**31 - 1, 2**32 + 7, 5 * 2**32 + 123])])
    for seed in (11, 23, 37, 12345):
        got = D.hash_values(torch, torch.from_numpy(idx.astype(np.int64)), seed).numpy()
        assert np.array_equal(got, O.hash_value(idx.astype(np.uint64), seed))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_sample_positions_follow_std_mt19937(tmp_path):
    n, samples = 1000, 64
    src = tmp_path / "mt.cpp"
    src.write_text(
        "#include <random>\n#include <cstdio>\n#include <set>\n#include <vector>\n"
        "int main(){int s=%d;std::vector<size_t> p={0,size_t(s-1),size_t(s-1)*s,size_t(s-1)*s+s-1};"
        "std::mt19937 rng(20261017+s);while(p.size()<%d){int r=rng()%%s,c=rng()%%s;p.push_back(r+size_t(c)*s);}"
        "std::set<size_t> u(p.begin(),p.end());for(auto v:u)std::printf(\"%%zu\\n\",v);}\n" % (n, samples))
    exe = tmp_path / "mt"
    subprocess.check_call(["g++", "-O1", "-o", str(exe), str(src)])
    want = [int(x) for x in subprocess.check_output([str(exe)]).split()]
    assert list(D.positions_for(n, samples)) == want


def _rows(path):
    with open(path) as f:
        return list(csv.reader(f))


@pytest.mark.gpu
@pytest.mark.parametrize("math_mode,size,depths", [("ffma", 256, "1,2"), ("3xtf32", 2048, "1")])
def test_driver_writes_reference_format(cuda, tmp_path, math_mode, size, depths):
    import bag_b200 as bag
    out = str(tmp_path / "run")
    rc = D.main(["--sizes", str(size), "--depths", depths, "--rounds", "1", "--target-ms", "5",
                 "--samples", "64", "--schedule", "batched", "--output", out, "--math", math_mode])
    bag.set_math_mode("ffma")
    assert rc == 0
    meta = json.load(open(out + ".metadata.json"))
    assert meta["sizes"] == [size] and meta["bag_math"] == math_mode
    assert isinstance(meta["cublas_version"], int) and meta["cublas_version"] >= 110000
    rounds = _rows(out + ".rounds.csv")
    assert rounds[0] == ["parent_n", "case", "mode", "round", "repeats", "batch_ms", "latency_ms",
                         "equivalent_tflops"]
    checks = _rows(out + ".correctness.csv")
    assert checks[0] == ["parent_n", "case", "repeats", "checked_values", "relative_l2_error",
                         "max_absolute_error", "max_scaled_error", "pass"]
    assert all(r[7] == "1" for r in checks[1:])
    cases = {r[1] for r in checks[1:]}
    assert "cublas_full" in cases and any(c.startswith("bag_column_minimal_d1") for c in cases)
    assert {r[1] for r in rounds[1:]} == cases
    ws = _rows(out + ".workspace.csv")
    assert ws[0] == ["parent_n", "depth", "basis", "bytes"] and len(ws) > 1


@pytest.mark.gpu
def test_profile_calls_runs_one_case_without_rounds(cuda, tmp_path, capsys):
    """--profile-calls K (strassen.cu:147-155): validation, then K calls of the
    one --only case inside cudaProfilerStart/Stop, and no timed rounds."""
    out = str(tmp_path / "prof")
    rc = D.main(["--sizes", "512", "--depths", "2", "--basis", "minimal", "--schedule", "batched",
                 "--only", "bag_column_minimal_d2_batched", "--profile-calls", "2",
                 "--output", out])
    assert rc == 0
    assert "PROFILE COMPLETE N=512 bag_column_minimal_d2_batched calls=2" in capsys.readouterr().out
    assert len(_rows(out + ".rounds.csv")) == 1            # header only
    checks = _rows(out + ".correctness.csv")
    assert {r[1] for r in checks[1:]} == {"bag_column_minimal_d2_batched"}


def test_profile_calls_needs_one_case():
    with pytest.raises(SystemExit):
        D.parse(["--profile-calls", "1"])


def test_depth_sweep_arguments():
    """The depth-sweep tool (measurement behind BAG_DEPTH_AUTO) parses square
    and rectangular shapes and rejects malformed ones, without a GPU."""
    from bag_b200 import depth_sweep as D
    args = D.parse_args(["--shapes", "4096,8192x4096x16384", "--depths", "1,2"])
    assert args.shapes == [(4096, 4096, 4096), (8192, 4096, 16384)]
    assert args.depths == [1, 2] and args.math == "3xtf32"
    for bad in ("0", "8x8", "axb", "8x8x-8"):
        with pytest.raises(ValueError):
            D.parse_shape(bad)
