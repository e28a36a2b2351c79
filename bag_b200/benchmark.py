"""Benchmark driver with the reference CUDA drivers' outputs.

    python -m bag_b200.benchmark --sizes 4096,8192 --depths 1,2 --basis both \\
        --schedule batched --math 3xtf32 --output results/bag_b200

Counterpart of the reference's ``benchmarks/cuda/bag.cu`` (options
``bag.cu:19-45``, cases ``bag.cu:72-100``, validation and timing
``bag.cu:104-127``) on this library, writing the same four files:

* ``<output>.metadata.json`` -- run description (``bag.cu:58-66``);
* ``<output>.rounds.csv`` -- ``parent_n,case,mode,round,repeats,batch_ms,latency_ms,equivalent_tflops``;
* ``<output>.correctness.csv`` -- ``parent_n,case,repeats,checked_values,relative_l2_error,max_absolute_error,max_scaled_error,pass``;
* ``<output>.workspace.csv`` -- ``parent_n,depth,basis,bytes``.

Cases per size N: ``cublas_full`` (cuBLAS FP32 through torch, TF32 off),
``strassen_column_four_batched`` (classic one level, ``bag_strassen_one_level``)
and ``bag_column_<basis>_d<depth>_<schedule>`` (``bag_matmul``, the reference
API: column-major ``C <- AB + C``), suffixed ``_3xtf32`` in that math mode.
Inputs are the reference's exactly representable hash values
(``fp32_baseline.cu:26-32``) with seeds 11, 23, 37 (+ seed offset); each case
is validated after 1 and 3 accumulating calls against an FP64 dot product at
sampled positions -- the four corners plus positions drawn from MT19937
seeded 20261017 + N, every position when N <= 128 -- and at sentinel positions
outside the product, with the reference's limits (relative L2 <= 3e-5,
max scaled error <= 1e-4; ``fp32_baseline.cu:121-192``).  Timing: CUDA events
around back-to-back calls, repeats adapted to ``--target-ms``, cases in a
shuffled order per round (``bag.cu:108-124``).

``--profile-calls K`` (with ``--only`` naming one case) is the counterpart of
the reference's ``benchmarks/cuda/strassen.cu:147-155``: after validation and
five warm-up calls it runs K calls between ``cudaProfilerStart`` and
``cudaProfilerStop`` and skips the timed rounds, so a profiler started with
``--profile-from-start off`` (``ncu``) sees exactly those K calls::

    ncu --profile-from-start off --clock-control none -k regex:leaf_pair -c 1 \
        python -m bag_b200.benchmark --sizes 4096 --depths 2 --basis minimal \
            --schedule batched --math 3xtf32 \
            --only bag_column_minimal_d2_batched_3xtf32 --profile-calls 1
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys

import numpy as np

SCHEDULES = ("serial", "seven", "batched")


def parse(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ints = lambda s: [int(x) for x in s.split(",") if x]  # noqa: E731
    p.add_argument("--sizes", type=ints, default=[1280, 1536, 1792, 2048])
    p.add_argument("--depths", type=ints, default=[1])
    p.add_argument("--basis", default="both", choices=["both", "minimal", "full"])
    p.add_argument("--schedule", default="all", choices=["all", *SCHEDULES])
    p.add_argument("--backend", default="column", choices=["column", "huge"])
    p.add_argument("--only", default="")
    p.add_argument("--seed-offset", type=int, default=0)
    p.add_argument("--rounds", type=int, default=5)
    p.add_argument("--target-ms", type=float, default=200.0)
    p.add_argument("--samples", type=int, default=128)
    p.add_argument("--output", default="results")
    p.add_argument("--validate-only", action="store_true")
    p.add_argument("--math", default="ffma", choices=["ffma", "3xtf32"])
    p.add_argument("--profile-calls", type=int, default=0,
                   help="run K calls of the --only case inside cudaProfilerStart/Stop, no rounds")
    o = p.parse_args(argv)
    for n in o.sizes:
        if n < 8 or n % 8:
            raise SystemExit("N must be positive and divisible by 8")
    for d in o.depths:
        if d < 1 or d > 8:
            raise SystemExit("depth must be 1..8")
    if o.rounds < 1 or o.target_ms <= 0 or o.samples < 16 or o.profile_calls < 0:
        raise SystemExit("invalid measurement options")
    if o.profile_calls and not o.only:
        raise SystemExit("profiling requires --only selecting one case")
    return o


# ---------------------------------------------------------------------------
# Inputs: the reference's exactly representable hash values.
# ---------------------------------------------------------------------------

_M32 = 0xFFFFFFFF


def _mix(x):
    x = x ^ (x >> 16)
    x = (x * 0x7FEB352D) & _M32
    x = x ^ (x >> 15)
    x = (x * 0x846CA68B) & _M32
    return x ^ (x >> 16)


def hash_values(torch, indices, seed: int):
    """value(i, seed) of fp32_baseline.cu:30-32 for an int64 tensor of indices."""
    x = ((indices & _M32) ^ (seed & _M32)) & _M32
    return ((_mix(x) & 65535) - 32768).to(torch.float32) * (1.0 / 65536.0)


def fill(torch, buf, seed: int) -> None:
    count = buf.numel()
    chunk = 1 << 26
    flat = buf.view(-1)
    for s in range(0, count, chunk):
        idx = torch.arange(s, min(count, s + chunk), device=buf.device, dtype=torch.int64)
        flat[s:s + idx.numel()] = hash_values(torch, idx, seed)


# ---------------------------------------------------------------------------
# Validation (sampled FP64 reference).
# ---------------------------------------------------------------------------

def positions_for(n: int, samples: int) -> np.ndarray:
    if n <= 128:
        return np.array([r + c * n for c in range(n) for r in range(n)], dtype=np.int64)
    pos = [0, n - 1, (n - 1) * n, (n - 1) * n + n - 1]
    mt = np.random.RandomState(20261017 + n)._bit_generator   # MT19937, init_genrand seeding
    while len(pos) < samples:
        row, col = (int(v) % n for v in mt.random_raw(2))
        pos.append(row + col * n)
    return np.unique(np.array(pos, dtype=np.int64))


def validate(torch, c, n: int, samples: int, repeats: int, seeds) -> dict:
    dev = c.device
    pos = positions_for(n, samples)
    rows, cols = pos % n, pos // n
    flat = c.view(-1)
    got = flat[torch.from_numpy(pos).to(dev)].double()
    # FP64 dots: A(row, k) at row + k*n, B(k, col) at k + col*n (column-major).
    ks = torch.arange(n, device=dev, dtype=torch.int64)
    dots = []
    for s in range(0, len(pos), 256):
        r = torch.from_numpy(rows[s:s + 256]).to(dev)[:, None]
        cc = torch.from_numpy(cols[s:s + 256]).to(dev)[:, None]
        x = hash_values(torch, r + ks[None, :] * n, seeds[0]).double()
        v = hash_values(torch, ks[None, :] + cc * n, seeds[1]).double()
        dots.append((x * v).sum(dim=1))
    dot = torch.cat(dots)
    ref = hash_values(torch, torch.from_numpy(pos).to(dev), seeds[2]).double() + repeats * dot
    # Sentinels: there are none outside an n x n product with ld = n.
    finite = bool(torch.isfinite(got).all())
    d = (got - ref).abs()
    rel = float(torch.sqrt((d * d).sum() / torch.clamp((ref * ref).sum(), min=1e-300)))
    max_abs = float(d.max())
    max_scaled = max_abs / (1.0 + float(ref.abs().max()))
    ok = finite and rel <= 3e-5 and max_scaled <= 1e-4
    return {"count": int(len(pos)), "relative_l2": rel, "max_abs": max_abs,
            "max_scaled": max_scaled, "pass": ok}


def cublas_version():
    """cuBLAS version as major*10000 + minor*100 + patch (cublasGetProperty), or None."""
    import ctypes
    import glob
    try:
        import torch
        root = os.path.dirname(os.path.dirname(torch.__file__))
        cands = sorted(glob.glob(os.path.join(root, "nvidia", "cublas", "lib", "libcublas.so*")))
        lib = ctypes.CDLL(cands[0] if cands else "libcublas.so")
        parts = []
        for prop in range(3):   # MAJOR_VERSION, MINOR_VERSION, PATCH_LEVEL
            v = ctypes.c_int(0)
            if lib.cublasGetProperty(prop, ctypes.byref(v)) != 0:
                return None
            parts.append(v.value)
        return parts[0] * 10000 + parts[1] * 100 + parts[2]
    except (OSError, AttributeError):
        return None


# ---------------------------------------------------------------------------
# The run.
# ---------------------------------------------------------------------------

def main(argv=None) -> int:
    o = parse(argv)
    import torch

    import bag_b200 as bag

    torch.backends.cuda.matmul.allow_tf32 = False
    bag.set_math_mode(o.math)
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream()
    backend = "column_tile64_k16_r4x8" if o.backend == "column" else "huge"
    suffix = "_3xtf32" if o.math == "3xtf32" else ""
    seeds = (11 + o.seed_offset, 23 + o.seed_offset, 37 + o.seed_offset)
    out_dir = os.path.dirname(o.output)
    if out_dir:
        os.makedirs(out_dir, exist_ok=True)
    props = torch.cuda.get_device_properties(dev)
    meta = {"gpu": props.name, "alpha": 1, "beta": 1,
            "math_mode": "CUBLAS_DEFAULT_MATH without TF32 (torch allow_tf32=False)",
            "seed_offset": o.seed_offset, "rounds": o.rounds, "target_ms": o.target_ms,
            "samples": o.samples, "backend": o.backend, "basis": o.basis,
            "schedule": o.schedule, "cuda_runtime": torch.version.cuda,
            "cublas_version": cublas_version(), "sizes": o.sizes, "depths": o.depths,
            "bag_math": o.math, "library": bag.lib().bag_version().decode()}
    with open(o.output + ".metadata.json", "w") as f:
        json.dump(meta, f)
    raw = open(o.output + ".rounds.csv", "w")
    checks = open(o.output + ".correctness.csv", "w")
    workspaces = open(o.output + ".workspace.csv", "w")
    raw.write("parent_n,case,mode,round,repeats,batch_ms,latency_ms,equivalent_tflops\n")
    checks.write("parent_n,case,repeats,checked_values,relative_l2_error,max_absolute_error,"
                 "max_scaled_error,pass\n")
    workspaces.write("parent_n,depth,basis,bytes\n")
    failed = False
    for n in o.sizes:
        a = torch.empty(n * n, device=dev)
        b = torch.empty(n * n, device=dev)
        c = torch.empty(n * n, device=dev)
        fill(torch, a, seeds[0])
        fill(torch, b, seeds[1])
        # Column-major n x n buffers: as row-major torch matrices they are the
        # transposes, so C_col = A_col B_col is c^T = (b^T a^T)^T, i.e. c += b @ a.
        am, bm, cm = a.view(n, n), b.view(n, n), c.view(n, n)
        cases = [("cublas_full", lambda: cm.addmm_(bm, am))]
        if bag.valid_shape(backend, n // 2):
            cases.append((f"strassen_{o.backend}_four_batched",
                          lambda: bag.strassen_one_level(a, b, c, n, backend, "four_batched_atomic")))
        keep = []
        for depth in o.depths:
            leaf, valid = n, True
            for _ in range(depth):
                valid = valid and leaf % 8 == 0 and leaf > 0
                leaf //= 2
            if not valid or not bag.valid_shape(backend, leaf):
                print(f"SKIP N={n} depth={depth} invalid leaf shape", flush=True)
                continue
            for basis in ("minimal", "full"):
                if o.basis not in ("both", basis):
                    continue
                ws = bag.Workspace(n, depth, basis)
                keep.append(ws)
                workspaces.write(f"{n},{depth},{basis},{ws.bytes()}\n")
                workspaces.flush()
                for sched in SCHEDULES:
                    if o.schedule not in ("all", sched):
                        continue
                    name = f"bag_{o.backend}_{basis}_d{depth}_{sched}{suffix}"
                    cases.append((name, (lambda w=ws, s=sched:
                                         bag.matmul(a, b, c, n, w, backend, s))))
        if o.only:
            keep_names = (o.only,) if o.profile_calls else (o.only, "cublas_full")
            cases = [x for x in cases if x[0] in keep_names]
        if len(cases) < (1 if o.profile_calls else 2):
            raise SystemExit("no legal BAG/Strassen case selected")
        for name, launch in cases:
            for repeats in (1, 3):
                fill(torch, c, seeds[2])
                for _ in range(repeats):
                    launch()
                torch.cuda.synchronize()
                e = validate(torch, c, n, o.samples, repeats, seeds)
                checks.write(f"{n},{name},{repeats},{e['count']},{e['relative_l2']!r},"
                             f"{e['max_abs']!r},{e['max_scaled']!r},{int(e['pass'])}\n")
                checks.flush()
                if not e["pass"]:
                    print(f"FP64 validation failed N={n} {name}", file=sys.stderr, flush=True)
                    failed = True
        print(f"N={n} FP64 {'FAIL' if failed else 'PASS'} cases={len(cases)}", flush=True)
        if failed or o.validate_only:
            continue
        if o.profile_calls:
            name, launch = cases[0]
            fill(torch, c, seeds[2])
            for _ in range(5):
                launch()
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStart()
            for _ in range(o.profile_calls):
                launch()
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStop()
            print(f"PROFILE COMPLETE N={n} {name} calls={o.profile_calls}", flush=True)
            continue
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

        def elapsed(launch, repeats):
            start.record(stream)
            for _ in range(repeats):
                launch()
            stop.record(stream)
            stop.synchronize()
            return start.elapsed_time(stop)

        for _, launch in cases:   # warm up
            fill(torch, c, seeds[2])
            p = elapsed(launch, 3) / 3
            elapsed(launch, max(3, min(10000, int(math.ceil(20.0 / max(p, 1e-4))))))
        order = np.arange(len(cases))
        shuffle = np.random.RandomState(20261017 + n)
        for rnd in range(o.rounds):
            shuffle.shuffle(order)
            for idx in order:
                name, launch = cases[idx]
                fill(torch, c, seeds[2])
                p = elapsed(launch, 3) / 3
                repeats = max(3, min(10000, int(math.ceil(o.target_ms / max(p, 1e-4)))))
                fill(torch, c, seeds[2])
                batch = elapsed(launch, repeats)
                ms = batch / repeats
                raw.write(f"{n},{name},endtoend,{rnd},{repeats},{batch!r},{ms!r},"
                          f"{2.0 * n * n * n / (ms * 1e9)!r}\n")
                raw.flush()
                print(f"{n} round={rnd} {name} ms={ms:.4f}", flush=True)
        del keep
    for f in (raw, checks, workspaces):
        f.close()
    if bag.device_error() != 0:
        print("device error word set", file=sys.stderr)
        return 1
    print(("FAILED " if failed else "COMPLETE ") + o.output, flush=True)
    return 1 if failed else 0


if __name__ == "__main__":
    sys.exit(main())
