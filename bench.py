#!/usr/bin/env python3
"""Benchmark of the B200-native BAG FP32 matmul (one JSON line on rank 0).

Workload: C = A @ B, FP32, M=N=K=16384, row-major, A then B
drawn N(0,1) from ``numpy.random.default_rng(2)``, two BAG recursion levels
(49 leaf products of 4096^3), Minimal basis.  A step is one
``C <- A@B + C`` call; inputs are 1 GiB each, larger than the 126 MB L2, so no
flush is needed between steps (``--config`` selects the other BASELINE
configs; those smaller than L2 are flushed).  The leaf arithmetic is ``--math``: 3xTF32
(default; tcgen05 tensor cores on hi/lo TF32 splits with FP32-folded chunks,
checked in the same run to stay within 1.25x the FFMA path's error, the
reference's numerics) or ffma (sequential FP32 fmaf chains, SIMT).

On N GPUs (one process per GPU, torchrun) the ranks form an R x S grid
(1x1, 2x1, 2x2, 4x2 for N = 1, 2, 4, 8): rank (i, j) owns row band i of every
one of the 2^depth block-rows of A and C and column band j of every block-column
of B and C.  BAG only combines blocks at equal offsets, so the recursion on
the compact (M/R) x K and K x (N/S) shards is exactly the restriction of the
full one: the units are independent, there is no collective on the data path,
and the total work is fixed (strong scaling).  ``e2e`` goes through the public
API from pinned host buffers: each rank uploads its A and B shards and reads
back its C shard.

``--impl reference`` times the reference algorithm's CPU restatement
(``oracle/bag_oracle.py``, numpy/OpenBLAS, all host threads) on a row-band
sample of the same workload -- the reference's only CPU path is its Triton
code under ``TRITON_INTERPRET=1``, which cannot run on the GPU box.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SIZE = 16384
DEPTH = 2
SEED = 2
METRIC = "effective FP32 TFLOP/s (2MNK/t) at N=16384 vs cuBLAS SGEMM, 1/2/4/8 B200"
WORKLOAD = ("cfg3: C=A@B FP32, M=N=K=16384 row-major, A,B ~ N(0,1) from default_rng(2), "
            "BAG depth 2 (49 leaf products of 4096^3), Minimal basis, C+=A@B per step")
# The BASELINE configs (A drawn before B from numpy.random.default_rng(seed),
# row-major).  cfg3 is the headline; the others are reproducible with --config.
CONFIGS = {
    "cfg1": dict(m=512, n=512, k=512, batch=1, depth=1, dist=("uniform", -1.0, 1.0), seed=0,
                 workload="cfg1: C=A@B FP32, M=N=K=512 row-major, A,B ~ U[-1,1) from "
                          "default_rng(0), BAG depth 1"),
    "cfg2": dict(m=4096, n=4096, k=4096, batch=1, depth=2, dist=("uniform", -1.0, 1.0), seed=1,
                 workload="cfg2: C=A@B FP32, M=N=K=4096 row-major, A,B ~ U[-1,1) from "
                          "default_rng(1), BAG depth 2 (--depth 1: one level)"),
    "cfg3": dict(m=SIZE, n=SIZE, k=SIZE, batch=1, depth=DEPTH, dist=("normal",), seed=SEED,
                 workload=WORKLOAD),
    "cfg4a": dict(m=8192, n=4096, k=16384, batch=1, depth=1, dist=("uniform", -1.0, 1.0), seed=3,
                  workload="cfg4a: C=A@B FP32, M=8192 K=16384 N=4096 row-major, A,B ~ U[-1,1) "
                           "from default_rng(3), BAG depth 1"),
    "cfg4b": dict(m=10000, n=10000, k=10000, batch=1, depth=1, dist=("uniform", -1.0, 1.0), seed=3,
                  workload="cfg4b: C=A@B FP32, M=N=K=10000 row-major (peeled), A,B ~ U[-1,1) "
                           "from default_rng(3), BAG depth 1"),
    "cfg5": dict(m=2048, n=2048, k=2048, batch=64, depth=1, dist=("uniform", 0.0, 1.0), seed=4,
                 workload="cfg5: 64 independent C=A@B FP32, 2048^3 row-major, A,B ~ U[0,1) from "
                          "default_rng(4), BAG depth 1 per problem, batch split over GPUs"),
}
CLOCK_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["bag", "reference"], default="bag")
    p.add_argument("--config", default="cfg3", choices=sorted(CONFIGS))
    p.add_argument("--size", type=int, default=None, help="square size (default: the config's)")
    p.add_argument("--depth", type=int, default=None, help="BAG depth (default: the config's)")
    p.add_argument("--basis", default="minimal", choices=["minimal", "full", "classic", "winograd"])
    p.add_argument("--math", default="3xtf32", choices=["3xtf32", "ffma"])
    p.add_argument("--cpu-seconds", type=float, default=12.0,
                   help="target CPU time of the bounded CPU-baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-comparators", action="store_true")
    args = p.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.size is not None:
        cfg.update(m=args.size, n=args.size, k=args.size)
    if args.depth is not None:
        cfg["depth"] = args.depth
    args.cfg = cfg
    args.depth = cfg["depth"]
    return args


# ---------------------------------------------------------------------------
# Inputs.
# ---------------------------------------------------------------------------

def make_inputs(cfg: dict) -> tuple[np.ndarray, np.ndarray]:
    """A (batch x) M x K then B (batch x) K x N from default_rng(seed)."""
    rng = np.random.default_rng(cfg["seed"])
    lead = (cfg["batch"],) if cfg["batch"] > 1 else ()
    shapes = (lead + (cfg["m"], cfg["k"]), lead + (cfg["k"], cfg["n"]))
    if cfg["dist"][0] == "normal":
        a, b = (rng.standard_normal(shp, dtype=np.float32) for shp in shapes)
    else:
        lo, hi = cfg["dist"][1:]
        a, b = (rng.uniform(lo, hi, shp).astype(np.float32) for shp in shapes)
    return a, b


def shard_grid(world: int) -> tuple[int, int]:
    """R x S rank grid: row bands x column bands."""
    return {1: (1, 1), 2: (2, 1), 4: (2, 2), 8: (4, 2)}.get(world, (world, 1))


def band_rows(size: int, depth: int, world: int, rank: int) -> np.ndarray:
    """Indices owned by band `rank` of `world`: its band of each of the 2^depth blocks."""
    blocks = 1 << depth
    q = size // blocks
    band = q // world
    return np.concatenate([np.arange(bi * q + rank * band, bi * q + (rank + 1) * band)
                           for bi in range(blocks)])


# ---------------------------------------------------------------------------
# Clock sampling during the timed region.
# ---------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi clock/throttle samples every 50 ms, each stamped with host time;
    summary() keeps those inside [window] (the timed region), else the nearest."""

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self._thread = None
        self.window: tuple[float, float] | None = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.device_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._thread = threading.Thread(target=self._read, daemon=True)
            self._thread.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self._thread is not None:
                self._thread.join(timeout=2)

    def summary(self) -> dict:
        sm, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = [ln for _, ln in self.lines]
        in_window = 0
        if self.window is not None and self.lines:
            t0, t1 = self.window
            inside = [ln for t, ln in self.lines if t0 <= t <= t1]
            in_window = len(inside)
            if inside:
                lines = inside
            else:   # timed region shorter than the sampling period: the nearest samples
                mid = 0.5 * (t0 + t1)
                lines = [ln for _, ln in sorted(self.lines, key=lambda x: abs(x[0] - mid))[:2]]
        for line in lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "samples_in_timed_region": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(maxes),
                "reasons": sorted(reasons), "samples": len(sm),
                "samples_in_timed_region": in_window}


# ---------------------------------------------------------------------------
# CPU baseline: the reference algorithm restated in numpy (oracle), timed on
# the host cores over a row-band sample of the workload.
# ---------------------------------------------------------------------------

def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        counts = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        if counts:
            return int(max(counts))
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_sample(a: np.ndarray, b: np.ndarray, depth: int, basis: str, units: int) -> tuple[float, float]:
    """Run the oracle BAG on `units` band rows of A with all of B (one problem) or
    on the first `units` problems (a batch); returns (seconds, flops)."""
    from oracle import bag_oracle as O
    if a.ndim == 3:
        t0 = time.perf_counter()
        for i in range(units):
            O.bag_product(a[i], b[i], depth, basis)
        dt = time.perf_counter() - t0
        return dt, 2.0 * units * a.shape[1] * a.shape[2] * b.shape[2]
    idx = band_rows(a.shape[0], depth, a.shape[0] // units, 0)
    a_s = np.ascontiguousarray(a[idx])
    t0 = time.perf_counter()
    O.bag_product(a_s, b, depth, basis)
    dt = time.perf_counter() - t0
    return dt, 2.0 * idx.size * b.shape[0] * b.shape[1]


def _sample_units(a: np.ndarray, depth: int) -> tuple[int, int]:
    """(first sample size, largest) in rows or problems."""
    if a.ndim == 3:
        return 1, a.shape[0]
    return max(a.shape[0] // 64, 16 << depth), a.shape[0]


def _describe_sample(a, b, units, depth, basis, dt) -> str:
    what = (f"{units} of the {a.shape[0]} {a.shape[1]}x{a.shape[2]}x{b.shape[2]} problems"
            if a.ndim == 3 else
            f"a {units}x{a.shape[1]} row-band shard of A times all of B ({b.shape[0]}x{b.shape[1]})")
    return (f"oracle/bag_oracle.py bag_product (numpy FP32, OpenBLAS leaves) on {what}, "
            f"depth {depth}, {basis} basis: {dt:.2f} s")


def cpu_baseline(a, b, depth, basis, target_s: float) -> dict:
    units, top = _sample_units(a, depth)
    dt, flops = cpu_sample(a, b, depth, basis, units)
    while dt < target_s / 3 and units * 2 <= top:
        units *= 2
        dt, flops = cpu_sample(a, b, depth, basis, units)
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": cpu_threads(), "kind": "port",
            "sample": _describe_sample(a, b, units, depth, basis, dt)}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    a, b = make_inputs(args.cfg)
    depth = args.depth
    units, top = _sample_units(a, depth)
    dt, _ = cpu_sample(a, b, depth, args.basis, units)
    while dt < args.cpu_seconds / 3 and units * 2 <= top:
        units *= 2
        dt, _ = cpu_sample(a, b, depth, args.basis, units)
    for _ in range(args.warmup):
        cpu_sample(a, b, depth, args.basis, units)
    times = []
    flops = 0.0
    for _ in range(args.steps):
        dt, flops = cpu_sample(a, b, depth, args.basis, units)
        times.append(dt)
    step = sum(times) / len(times)
    value = flops / step / 1e12
    base = {"value": value, "unit": "TFLOP/s", "cores": cpu_threads(), "kind": "port",
            "sample": _describe_sample(a, b, units, depth, args.basis, step)}
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": step * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.cfg["workload"], "sample_units": units, "depth": depth,
                       "basis": args.basis, "parallelism": "host threads (BLAS)"},
            "cpu_baseline": base,
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# The GPU arm.
# ---------------------------------------------------------------------------

def run_bag(args) -> None:
    import torch
    import torch.distributed as dist

    import bag_b200 as bag

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    torch.backends.cuda.matmul.allow_tf32 = False
    bag.set_math_mode(args.math)

    cfg, depth = args.cfg, args.depth
    M, N, K, batch = cfg["m"], cfg["n"], cfg["k"], cfg["batch"]
    gr, gc = shard_grid(world)
    a_np, b_np = make_inputs(cfg)
    if batch > 1:
        # A batch: every rank takes batch/world whole problems.
        if batch % world:
            raise SystemExit("the batch must split evenly over the GPUs")
        nb = batch // world
        a_shard = np.ascontiguousarray(a_np[rank * nb:(rank + 1) * nb])
        b_shard = np.ascontiguousarray(b_np[rank * nb:(rank + 1) * nb])
        mg, ng = M, N
        parallelism = f"batch split, {nb} problems per GPU"
    else:
        if M % ((4 << depth) * gr) or N % ((4 << depth) * gc):
            raise SystemExit("the problem must split into aligned bands for this GPU count")
        nb = 1
        rows = band_rows(M, depth, gr, rank // gc)
        cols = band_rows(N, depth, gc, rank % gc)
        mg, ng = rows.size, cols.size
        a_shard = np.ascontiguousarray(a_np[rows]) if gr > 1 else a_np
        b_shard = np.ascontiguousarray(b_np[:, cols]) if gc > 1 else b_np
        parallelism = f"{gr}x{gc} grid of row/column-band shards"
    lead = (nb,) if batch > 1 else ()

    # Pinned host buffers (the e2e inputs) and device buffers (the value inputs).
    a_host = torch.from_numpy(a_shard).pin_memory()
    b_host = torch.from_numpy(b_shard).pin_memory()
    c_host = torch.empty(lead + (mg, ng), dtype=torch.float32).pin_memory()
    a_dev = a_host.to(device)
    b_dev = b_host.to(device)
    c_dev = torch.zeros(lead + (mg, ng), dtype=torch.float32, device=device)
    del a_np
    # Row-major C(mg x ng) = A B is the column-major ng x mg problem.
    ws = bag.Workspace.for_problem(ng, mg, K, depth, args.basis, batch=nb)
    stream = torch.cuda.current_stream()
    gemm = bag.sgemm_batched if batch > 1 else bag.sgemm

    def step():
        gemm(a_dev, b_dev, c_dev, beta=1.0, depth=depth, basis=args.basis, workspace=ws)

    def barrier():
        if world > 1:
            dist.barrier()

    def reduce_max(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def reduce_sum(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    # Leaf-kernel events, created up front (torch creates events lazily).
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(args.steps)]
    # Phase events per step: before the call, after its materialisation
    # launches, after its last launch (with the leaf pair: stages | prepare |
    # leaves | decode).
    phases = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3))
              for _ in range(args.steps)]
    for ev in [e for p in pairs for e in p] + [e for p in phases for e in p]:
        ev.record()
    torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    # Inputs smaller than twice the 126 MB L2 (cfg1, cfg2) get an L2 flush
    # (a 256 MiB write) before every timed step, outside its events; larger
    # ones are timed back to back.
    input_bytes = 4 * (a_shard.size + b_shard.size)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=device) if input_bytes < (256 << 20) \
        else None
    launches0 = bag.launch_count()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    step_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        time.sleep(0.15)   # let the sampler start before the timed region
        host0 = time.time()
        t_start.record()
        for i in range(args.steps):
            if flush is not None:
                flush.fill_(float(i))
                step_events[i][0].record()
            bag.profile_events(*pairs[i])
            bag.profile_phase_events(phases[i][1], phases[i][2])
            phases[i][0].record()
            step()
            if flush is not None:
                step_events[i][1].record()
        bag.profile_events(None, None)
        bag.profile_phase_events(None, None)
        t_end.record()
        torch.cuda.synchronize()
        clocks.window = (host0, time.time())
        time.sleep(0.12)
    barrier()
    launches = reduce_sum(bag.launch_count() - launches0)
    leaf_path = bag.last_leaf_path()
    leaf_kernel = bag.last_leaf_kernel()
    if flush is not None:
        ms = reduce_max(sum(s0.elapsed_time(s1) for s0, s1 in step_events)) / args.steps
        l2_note = "inputs smaller than L2: a 256 MiB buffer written before each timed step"
    else:
        ms = reduce_max(t_start.elapsed_time(t_end)) / args.steps
        l2_note = f"inputs larger than L2 ({input_bytes / 2**30:.2f} GiB per GPU); no flush"
    del flush
    leaf_ms = reduce_max(sum(s.elapsed_time(e) for s, e in pairs) / args.steps)

    def phase_mean(f):
        return reduce_max(sum(f(i) for i in range(args.steps)) / args.steps)

    # Each phase includes the launch gap in front of it.
    phases_ms = {
        "stages": phase_mean(lambda i: phases[i][0].elapsed_time(phases[i][1])),
        "prepare": phase_mean(lambda i: phases[i][1].elapsed_time(pairs[i][0])),
        "leaves": leaf_ms,
        "decode": phase_mean(lambda i: pairs[i][1].elapsed_time(phases[i][2])),
        "call": phase_mean(lambda i: phases[i][0].elapsed_time(phases[i][2])),
    }
    flops_total = 2.0 * M * N * K * batch
    value = flops_total / (ms * 1e-3) / 1e12
    # Executed leaf FLOPs of this rank's launch: nb x 7^depth products of
    # (mg/2^d)(ng/2^d)(K/2^d) (ragged extents peel into strips of plain work).
    f_exec = nb * 7 ** depth * 2.0 * (mg / 2 ** depth) * (ng / 2 ** depth) * (K / 2 ** depth)
    leaf_tflops = f_exec / (leaf_ms * 1e-3) / 1e12

    # FP32 FFMA peak: nominal at the max SM clock, and measured by the probe.
    props = torch.cuda.get_device_properties(device)
    sms = props.multi_processor_count
    csum = clocks.summary()
    max_mhz = csum["sm_max_mhz"] or 1965.0
    nominal = sms * 128 * 2 * max_mhz * 1e6 / 1e12
    sink = torch.empty(sms * 1024, dtype=torch.float32, device=device)
    import ctypes
    fl = ctypes.c_double(0)
    for _ in range(2):
        bag._check(bag.lib().bag_ffma_probe(sink.data_ptr(), 20000, stream.cuda_stream,
                                            ctypes.byref(fl)))
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    bag._check(bag.lib().bag_ffma_probe(sink.data_ptr(), 20000, stream.cuda_stream,
                                        ctypes.byref(fl)))
    p1.record()
    torch.cuda.synchronize()
    probe = fl.value / (p0.elapsed_time(p1) * 1e-3) / 1e12

    # End to end through the public API, host buffers in and out, pipelined
    # like a serving loop: step i+1's inputs are uploaded on one copy stream
    # while step i computes, and step i's C is read back on another while
    # step i+1 computes (two device and two pinned-host buffer sets).  Every
    # step still moves its own inputs host->device and its result back.
    comp = torch.cuda.current_stream()
    h2d_s, d2h_s = torch.cuda.Stream(device), torch.cuda.Stream(device)
    a2 = [a_dev, torch.empty_like(a_dev)]
    b2 = [b_dev, torch.empty_like(b_dev)]
    c2 = [c_dev, torch.empty_like(c_dev)]
    ch2 = [c_host, torch.empty(c_host.shape, dtype=torch.float32, pin_memory=True)]
    up_done = [torch.cuda.Event(), torch.cuda.Event()]
    comp_done = [torch.cuda.Event(), torch.cuda.Event()]
    down_done = [torch.cuda.Event(), torch.cuda.Event()]

    def e2e_run(steps: int, start_event=None) -> int:
        if start_event is not None:
            h2d_s.wait_event(start_event)
        for i in range(steps):
            sl = i % 2
            with torch.cuda.stream(h2d_s):
                if i >= 2:
                    h2d_s.wait_event(comp_done[sl])   # step i-2 no longer reads slot sl
                a2[sl].copy_(a_host, non_blocking=True)
                b2[sl].copy_(b_host, non_blocking=True)
                up_done[sl].record(h2d_s)
            comp.wait_event(up_done[sl])
            if i >= 2:
                comp.wait_event(down_done[sl])        # step i-2's C has been read back
            gemm(a2[sl], b2[sl], c2[sl], beta=0.0, depth=depth, basis=args.basis, workspace=ws)
            comp_done[sl].record(comp)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(comp_done[sl])
                ch2[sl].copy_(c2[sl], non_blocking=True)
                down_done[sl].record(d2h_s)
        comp.wait_stream(h2d_s)
        comp.wait_stream(d2h_s)
        return (steps - 1) % 2

    # The timed run starts and ends with an empty pipeline (the first upload
    # and the last read-back overlap nothing), so it runs at least 20 steps to
    # report a serving loop's steady rate; PCIe bounds it (~52 GB/s each way
    # on these boxes: 2 GB up and 1 GB down per cfg3 step take ~42.6 ms).
    e2e_steps = max(args.steps, 20)
    e2e_run(2)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    last = e2e_run(e2e_steps, start_event=e0)
    e1.record(comp)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = reduce_max(e0.elapsed_time(e1)) / e2e_steps
    c_res = c2[last]   # this run's final C = A@B, for the accuracy check
    h2d = int(reduce_sum(4.0 * (a_shard.size + b_shard.size)))   # all ranks' shards
    d2h = 4 * M * N * batch

    # Comparators: cuBLAS SGEMM (torch, IEEE FP32, no TF32) and this library's
    # FFMA path on the same inputs.
    comparators = {}
    if rank == 0 and world == 1 and not args.no_comparators and leaf_path != "ffma":
        bag.set_math_mode("ffma")
        c_tmp = torch.zeros_like(c_dev)   # c_dev keeps the e2e result for the accuracy check

        def ffma_step():
            gemm(a_dev, b_dev, c_tmp, beta=1.0, depth=depth, basis=args.basis, workspace=ws)

        for _ in range(2):
            ffma_step()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for _ in range(args.steps):
            ffma_step()
        f1.record()
        torch.cuda.synchronize()
        del c_tmp
        fms = f0.elapsed_time(f1) / args.steps
        comparators["bag_ffma_path"] = {"tflops": flops_total / (fms * 1e-3) / 1e12,
                                        "ms_per_step": fms,
                                        "how": "same call, bag_set_math_mode(BAG_MATH_FFMA)"}
        bag.set_math_mode(args.math)
    if rank == 0 and world == 1 and not args.no_comparators:
        c_cmp = torch.zeros_like(c_dev)

        def cublas_step():
            if batch > 1:
                c_cmp.baddbmm_(a_dev, b_dev)
            else:
                c_cmp.addmm_(a_dev, b_dev)

        for _ in range(2):
            cublas_step()
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        for _ in range(args.steps):
            cublas_step()
        c1.record()
        torch.cuda.synchronize()
        cms = c0.elapsed_time(c1) / args.steps
        comparators["cublas_sgemm_fp32"] = {"tflops": flops_total / (cms * 1e-3) / 1e12,
                                            "ms_per_step": cms,
                                            "how": "torch addmm_/baddbmm_, allow_tf32=False "
                                                   "(cuBLAS FP32)"}
        del c_cmp

    # Accuracy of this run's result (the last e2e step computed C = A@B once)
    # and, for the tensor path, of the FFMA path -- the reference's numerics --
    # on the same inputs at the same depth: the bound is <= 1.25x that and <= 1e-4.
    accuracy = {}
    if rank == 0 and world == 1:
        c = c_res
        c_ffma = None
        if leaf_path != "ffma":
            bag.set_math_mode("ffma")
            c_ffma = torch.zeros_like(c_dev)
            gemm(a_dev, b_dev, c_ffma, beta=0.0, depth=depth, basis=args.basis, workspace=ws)
            bag.set_math_mode(args.math)
        # FP64 reference on the GPU (cuBLAS DGEMM), per problem in column panels.
        panel = 2048
        num = num_f = den = 0.0
        for i in range(nb):
            ai, bi, ci = (a_dev[i], b_dev[i], c[i]) if batch > 1 else (a_dev, b_dev, c)
            fi = None if c_ffma is None else (c_ffma[i] if batch > 1 else c_ffma)
            a64 = ai.double()
            for j in range(0, ng, panel):
                ref = a64 @ bi[:, j:j + panel].double()
                diff = ci[:, j:j + panel].double() - ref
                num += float((diff * diff).sum())
                den += float((ref * ref).sum())
                if fi is not None:
                    diff = fi[:, j:j + panel].double() - ref
                    num_f += float((diff * diff).sum())
            del a64
        accuracy = {"rel_frobenius_vs_fp64": (num / den) ** 0.5}
        if c_ffma is not None:
            ffma_err = (num_f / den) ** 0.5
            accuracy.update({"ffma_path_rel_frobenius_vs_fp64": ffma_err,
                             "ratio_to_ffma_path": accuracy["rel_frobenius_vs_fp64"] / ffma_err,
                             "bound": "<= 1.25x the FFMA path (sequential fmaf leaves, the "
                                      "reference CUDA numerics) and <= 1e-4",
                             "within_bound": accuracy["rel_frobenius_vs_fp64"] <= min(
                                 1.25 * ffma_err, 1e-4)})
            del c_ffma

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(a_host.numpy(), b_np, depth, args.basis, args.cpu_seconds)

    if rank == 0:
        if leaf_path == "3xtf32":
            peaks = measured_peaks()
            tf32 = peaks.get("bf16_tflops", 1590.0) / 2.0
            sustained = peaks.get("bf16_tflops_sustained", 1400.0) / 2.0
            # The workspace was created in 3xTF32 mode, so the call runs the
            # prepare pass (prep_group_kernel), the leaf kernel on the prepared
            # operands and, at depth 2, the deferred decode; the leaf events
            # bracket the leaf launches only ("prepare_and_materialise_ms" is
            # the rest of the call).
            kernels = {
                "tf32_pair": ("leaf_pair_kernel (3xTF32 tcgen05.mma.cta_group::2, 256x256 tiles "
                              "on SM pairs, prepared TF32 hi/lo operands)",
                              "leaf_pair_cfg3_traffic.txt"),
                "tf32_single": ("leaf_prep_kernel<256> (3xTF32 tcgen05, 128x256 tiles per SM, "
                                "prepared TF32 hi/lo operands)", "leaf_prep_cfg3_traffic.txt"),
                "tf32_fused": ("leaf_tc_kernel (3xTF32 tcgen05, transforms in the prologue)",
                               "leaf_tc_cfg3_traffic.txt"),
            }
            kname, kfile = kernels.get(leaf_kernel, kernels["tf32_fused"])
            roofline = {"bound": "tensor", "kernel": kname,
                        "achieved": leaf_tflops, "peak": tf32 / 3.0, "unit": "TFLOP/s",
                        "frac": leaf_tflops / (tf32 / 3.0),
                        "traffic": read_traffic(kfile),
                        "prepare_and_materialise_ms": ms - leaf_ms,
                        "peak_source": "MEASURED_PEAKS.json bf16_tflops (burst, of measured) / 2 "
                                       "(dense TF32 = half the bf16 rate) / 3 (three MMAs per "
                                       "leaf product: hi*hi, hi*lo, lo*hi)",
                        "frac_of_sustained": leaf_tflops / (sustained / 3.0),
                        "leaf_ms": leaf_ms, "algorithmic_flops_per_launch": f_exec}
        else:
            roofline = {"bound": "compute", "kernel": "leaf_gemm_kernel (FP32 FFMA SIMT)",
                        "achieved": leaf_tflops, "peak": nominal, "unit": "TFLOP/s",
                        "frac": leaf_tflops / nominal,
                        "traffic": read_traffic("leaf_gemm_cfg3_traffic.txt"),
                        "peak_source": f"nominal FP32 FFMA {sms} SM x 128 lanes x 2 x "
                                       f"{max_mhz:.0f} MHz (MEASURED_PEAKS.json has no FP32 "
                                       f"SIMT figure)",
                        "ffma_probe_tflops": probe, "frac_of_probe": leaf_tflops / probe,
                        "leaf_ms": leaf_ms, "algorithmic_flops_per_launch": f_exec}
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": cfg["workload"], "M": M, "N": N, "K": K, "batch": batch,
                       "depth": depth, "basis": args.basis, "layout": "row-major",
                       "leaf_math": leaf_path, "l2": l2_note,
                       "parallelism": parallelism if world > 1 else "single GPU"},
            "e2e": {"value": flops_total / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                    "steps": e2e_steps,
                    "how": "public sgemm API from pinned host buffers; uploads of step i+1 and "
                           "the read-back of step i overlap step i's compute (2 buffer sets)"},
            "roofline": roofline,
            "ffma_probe_tflops": probe,
            "clocks": {k: csum[k] for k in ("sm_mhz", "sm_max_mhz", "reasons",
                                            "samples_in_timed_region")},
            "gpu_launches": int(launches),
            "phases_ms": phases_ms,
            "executed_tflops": f_exec * world / (ms * 1e-3) / 1e12,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if comparators:
            line["comparators"] = comparators
        if accuracy:
            line["accuracy"] = accuracy
        print(json.dumps(line), flush=True)
    del ws
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def measured_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def read_traffic(name: str):
    """DRAM bytes per leaf launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_full_launch:"):
                    fields = line.split(":", 1)[1].split()
                    return float(fields[0]) if fields else None
    except (OSError, ValueError):
        pass
    return None


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_bag(args)


if __name__ == "__main__":
    main()
