#!/usr/bin/env python3
"""Benchmark of the B200-native BAG FP32 matmul (one JSON line on rank 0).

Workload: C = A @ B, FP32, M=N=K=16384, row-major, A then B
drawn N(0,1) from ``numpy.random.default_rng(2)``, two BAG recursion levels
(49 leaf products of 4096^3), Minimal basis.  A step is one
``C <- A@B + C`` call; inputs are 1 GiB each, larger than the 126 MB L2, so no
flush is needed between steps.  The leaf arithmetic is ``--math``: 3xTF32
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
CLOCK_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["bag", "reference"], default="bag")
    p.add_argument("--size", type=int, default=SIZE)
    p.add_argument("--depth", type=int, default=DEPTH)
    p.add_argument("--basis", default="minimal", choices=["minimal", "full", "classic"])
    p.add_argument("--math", default="3xtf32", choices=["3xtf32", "ffma"])
    p.add_argument("--cpu-seconds", type=float, default=12.0,
                   help="target CPU time of the bounded CPU-baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-comparators", action="store_true")
    return p.parse_args()


# ---------------------------------------------------------------------------
# Inputs.
# ---------------------------------------------------------------------------

def make_inputs(size: int) -> tuple[np.ndarray, np.ndarray]:
    rng = np.random.default_rng(SEED)
    a = rng.standard_normal((size, size), dtype=np.float32)
    b = rng.standard_normal((size, size), dtype=np.float32)
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


def cpu_sample(a: np.ndarray, b: np.ndarray, depth: int, basis: str, rows: int) -> tuple[float, float]:
    """Run the oracle BAG on `rows` band rows of A (all of B); returns (seconds, flops)."""
    from oracle import bag_oracle as O
    idx = band_rows(a.shape[0], depth, a.shape[0] // rows, 0)
    a_s = np.ascontiguousarray(a[idx])
    t0 = time.perf_counter()
    O.bag_product(a_s, b, depth, basis)
    dt = time.perf_counter() - t0
    return dt, 2.0 * rows * b.shape[0] * b.shape[1]


def cpu_baseline(a, b, depth, basis, target_s: float) -> dict:
    size = a.shape[0]
    rows = max(size // 64, 16 << depth)
    dt, flops = cpu_sample(a, b, depth, basis, rows)
    while dt < target_s / 3 and rows * 2 <= size:
        rows *= 2
        dt, flops = cpu_sample(a, b, depth, basis, rows)
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": cpu_threads(), "kind": "port",
            "sample": f"oracle/bag_oracle.py bag_product (numpy FP32, OpenBLAS leaves) on a "
                      f"{rows}x{size} row-band shard of A times all of B ({size}x{size}), "
                      f"depth {depth}, {basis} basis: {dt:.2f} s"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    a, b = make_inputs(args.size)
    size, depth = args.size, args.depth
    rows = max(size // 64, 16 << depth)
    dt, _ = cpu_sample(a, b, depth, args.basis, rows)
    while dt < args.cpu_seconds / 3 and rows * 2 <= size:
        rows *= 2
        dt, _ = cpu_sample(a, b, depth, args.basis, rows)
    for _ in range(args.warmup):
        cpu_sample(a, b, depth, args.basis, rows)
    times = []
    flops = 0.0
    for _ in range(args.steps):
        dt, flops = cpu_sample(a, b, depth, args.basis, rows)
        times.append(dt)
    step = sum(times) / len(times)
    value = flops / step / 1e12
    base = {"value": value, "unit": "TFLOP/s", "cores": cpu_threads(), "kind": "port",
            "sample": f"oracle/bag_oracle.py bag_product (numpy FP32, OpenBLAS leaves) on a "
                      f"{rows}x{size} row-band shard of A times all of B, depth {depth}"}
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": step * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "sample_rows": rows, "depth": depth,
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

    size, depth = args.size, args.depth
    gr, gc = shard_grid(world)
    if size % ((4 << depth) * gr) or size % ((4 << depth) * gc):
        raise SystemExit("size must split into aligned bands for this GPU count")
    a_np, b_np = make_inputs(size)
    rows = band_rows(size, depth, gr, rank // gc)
    cols = band_rows(size, depth, gc, rank % gc)
    mg, ng = rows.size, cols.size
    a_shard = np.ascontiguousarray(a_np[rows])
    b_shard = np.ascontiguousarray(b_np[:, cols]) if gc > 1 else b_np

    # Pinned host buffers (the e2e inputs) and device buffers (the value inputs).
    a_host = torch.from_numpy(a_shard).pin_memory()
    b_host = torch.from_numpy(b_shard).pin_memory()
    c_host = torch.empty((mg, ng), dtype=torch.float32).pin_memory()
    a_dev = a_host.to(device)
    b_dev = b_host.to(device)
    c_dev = torch.zeros((mg, ng), dtype=torch.float32, device=device)
    del a_np
    # Row-major C(mg x ng) = A B is the column-major ng x mg problem.
    ws = bag.Workspace.for_problem(ng, mg, size, depth, args.basis)
    stream = torch.cuda.current_stream()

    def step():
        bag.sgemm(a_dev, b_dev, c_dev, beta=1.0, depth=depth, basis=args.basis, workspace=ws)

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
    for s, e in pairs:
        s.record()
        e.record()
    torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches0 = bag.launch_count()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        time.sleep(0.15)   # let the sampler start before the timed region
        host0 = time.time()
        t_start.record()
        for i in range(args.steps):
            bag.profile_events(*pairs[i])
            step()
        bag.profile_events(None, None)
        t_end.record()
        torch.cuda.synchronize()
        clocks.window = (host0, time.time())
        time.sleep(0.12)
    barrier()
    launches = reduce_sum(bag.launch_count() - launches0)
    leaf_path = bag.last_leaf_path()
    ms = reduce_max(t_start.elapsed_time(t_end)) / args.steps
    leaf_ms = reduce_max(sum(s.elapsed_time(e) for s, e in pairs) / args.steps)
    flops_total = 2.0 * size * size * size
    value = flops_total / (ms * 1e-3) / 1e12
    # Executed leaf FLOPs of this rank's launch: 7^depth products of (mg/2^d)(ng/2^d)(K/2^d).
    f_exec = 7 ** depth * 2.0 * (mg / 2 ** depth) * (ng / 2 ** depth) * (size / 2 ** depth)
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

    # End to end through the public API, host buffers in and out.
    def e2e_step():
        a_dev.copy_(a_host, non_blocking=True)
        b_dev.copy_(b_host, non_blocking=True)
        bag.sgemm(a_dev, b_dev, c_dev, beta=0.0, depth=depth, basis=args.basis, workspace=ws)
        c_host.copy_(c_dev, non_blocking=True)

    for _ in range(min(args.warmup, 2)):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = reduce_max(e0.elapsed_time(e1)) / args.steps
    h2d = int(reduce_sum(4.0 * (mg * size + size * ng)))   # all ranks' shards
    d2h = 4 * size * size

    # Comparators: cuBLAS SGEMM (torch, IEEE FP32, no TF32) and this library's
    # FFMA path on the same inputs.
    comparators = {}
    if rank == 0 and world == 1 and not args.no_comparators and leaf_path != "ffma":
        bag.set_math_mode("ffma")
        c_tmp = torch.zeros_like(c_dev)   # c_dev keeps the e2e result for the accuracy check

        def ffma_step():
            bag.sgemm(a_dev, b_dev, c_tmp, beta=1.0, depth=depth, basis=args.basis, workspace=ws)

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
        a_full = a_dev
        c_cmp = torch.zeros((size, size), dtype=torch.float32, device=device)
        for _ in range(2):
            c_cmp.addmm_(a_full, b_dev)
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        for _ in range(args.steps):
            c_cmp.addmm_(a_full, b_dev)
        c1.record()
        torch.cuda.synchronize()
        cms = c0.elapsed_time(c1) / args.steps
        comparators["cublas_sgemm_fp32"] = {"tflops": flops_total / (cms * 1e-3) / 1e12,
                                            "ms_per_step": cms,
                                            "how": "torch addmm_, allow_tf32=False (cuBLAS FP32)"}
        del c_cmp

    # Accuracy of this run's result (the last e2e step computed C = A@B once)
    # and, for the tensor path, of the FFMA path -- the reference's numerics --
    # on the same inputs at the same depth: the bound is <= 1.25x that and <= 1e-4.
    accuracy = {}
    if rank == 0 and world == 1:
        c = c_dev
        c_ffma = None
        if leaf_path != "ffma":
            bag.set_math_mode("ffma")
            c_ffma = torch.zeros_like(c_dev)
            bag.sgemm(a_dev, b_dev, c_ffma, beta=0.0, depth=depth, basis=args.basis, workspace=ws)
            bag.set_math_mode(args.math)
        # FP64 reference on the GPU (cuBLAS DGEMM), column panels to bound memory.
        panel = 2048
        num = num_f = den = 0.0
        a64 = a_dev.double()
        for j in range(0, size, panel):
            ref = a64 @ b_dev[:, j:j + panel].double()
            diff = c[:, j:j + panel].double() - ref
            num += float((diff * diff).sum())
            den += float((ref * ref).sum())
            if c_ffma is not None:
                diff = c_ffma[:, j:j + panel].double() - ref
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
            # prepare pass (prep_kernel) and then leaf_prep_kernel; the leaf
            # events bracket the leaf launches only.
            roofline = {"bound": "tensor",
                        "kernel": "leaf_prep_kernel<256> (3xTF32 tcgen05 on prepared TF32 hi/lo operands)",
                        "achieved": leaf_tflops, "peak": tf32 / 3.0, "unit": "TFLOP/s",
                        "frac": leaf_tflops / (tf32 / 3.0),
                        "traffic": read_traffic("leaf_prep_cfg3_traffic.txt"),
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
            "config": {"workload": WORKLOAD, "M": size, "N": size, "K": size, "depth": depth,
                       "basis": args.basis, "layout": "row-major", "leaf_math": leaf_path,
                       "l2": "inputs larger than L2 (1 GiB each); no flush",
                       "parallelism": f"{gr}x{gc} grid of row/column-band shards" if world > 1
                       else "single GPU"},
            "e2e": {"value": flops_total / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "roofline": roofline,
            "ffma_probe_tflops": probe,
            "clocks": {k: csum[k] for k in ("sm_mhz", "sm_max_mhz", "reasons",
                                            "samples_in_timed_region")},
            "gpu_launches": int(launches),
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
                    return float(line.split(":", 1)[1])
    except OSError:
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
