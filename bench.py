#!/usr/bin/env python3
"""Benchmark of the B200-native BAG FP32 matmul (one JSON line on rank 0).

Workload: C = A @ B, FP32, M=N=K=16384, row-major, A then B
drawn N(0,1) from ``numpy.random.default_rng(2)``, two BAG recursion levels
(49 leaf products of 4096^3), Minimal basis.  A step is one
``C <- A@B + C`` call; inputs are 1 GiB each, larger than the 126 MB L2, so no
flush is needed between steps (``--config`` selects the other BASELINE
configs; those smaller than L2 are flushed).  The leaf arithmetic is ``--math``: 3xTF32
(default; tcgen05 tensor cores on hi/lo TF32 splits with FP32-folded chunks)
or ffma (sequential FP32 fmaf chains, SIMT).  After the timed region the run
checks its own result: relative Frobenius error against an FP64 GEMM, within
1.25x the reference CUDA BAG's error on the same inputs (median of 3 runs of
the reference's own kernel, compiled from its headers) and within 1e-4.

On N GPUs (one process per GPU, torchrun) the ranks form an R x S grid
(1x1, 2x1, 2x2, 4x2 for N = 1, 2, 4, 8): rank (i, j) owns row band i of every
one of the 2^depth block-rows of A and C and column band j of every block-column
of B and C.  BAG only combines blocks at equal offsets, so the recursion on
the compact (M/R) x K and K x (N/S) shards is exactly the restriction of the
full one: the units are independent, there is no collective on the compute
path, and the total work is fixed (strong scaling).  ``e2e`` goes through the
public API from pinned host buffers and moves every host byte once: rank
(i, j) uploads 1/S of its A shard and 1/R of its B shard, NCCL all-gathers
assemble the shards inside the row and column groups over NVLink, and each
rank reads back its own C shard.  ``e2e_from_gpu0`` (N > 1) times the
one-process entry point ``bag_sgemm_multi`` with A, B and C on GPU 0.

``--impl reference`` times the reference algorithm's CPU restatement
(``oracle/bag_oracle.py``, numpy/OpenBLAS, every host core) on a row-band
sample of the same workload, with an FP64 numpy classical GEMM on the same
sample beside it.
"""

from __future__ import annotations

import argparse
import ctypes
import glob
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
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libbagref.so")
SOAK_S = 1.0          # untimed steps before the timed region, so every N starts power-steady


def parse_args(argv=None):
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
    args = p.parse_args(argv)
    if args.warmup < 1 or args.steps < 1:
        p.error("--steps and --warmup must be positive")
    cfg = dict(CONFIGS[args.config])
    if args.size is not None:
        cfg.update(m=args.size, n=args.size, k=args.size)
    if args.depth is not None:
        cfg["depth"] = args.depth
    args.cfg = cfg
    args.depth = cfg["depth"]
    return args


# ---------------------------------------------------------------------------
# Inputs and the shard layout.
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


def upload_pieces(shard_rows_a: int, k: int, gr: int, gc: int, rank: int) -> dict:
    """Which slice of its shards rank (i, j) uploads from the host in ``e2e``.

    The A shard (shard_rows_a x k) is shared by the S ranks of row group i:
    rank (i, j) uploads its rows [j*pa, (j+1)*pa).  The B shard (k x n_shard)
    is shared by the R ranks of column group j: rank (i, j) uploads its rows
    [i*pb, (i+1)*pb).  An all-gather inside each group (ranks in grid order)
    then assembles both shards, so every host byte crosses PCIe once."""
    i, j = divmod(rank, gc)
    if shard_rows_a % gc or k % gr:
        raise ValueError("the shards do not split evenly over the row and column groups")
    pa, pb = shard_rows_a // gc, k // gr
    return {"a_rows": (j * pa, (j + 1) * pa), "b_rows": (i * pb, (i + 1) * pb),
            "row_group": [i * gc + jj for jj in range(gc)],
            "col_group": [ii * gc + j for ii in range(gr)]}


def line_config(args, world: int) -> dict:
    """The workload description both arms print (the driver compares them)."""
    cfg = args.cfg
    gr, gc = shard_grid(world)
    batch = cfg["batch"]
    if batch > 1:
        per_gpu = 4 * (batch // max(world, 1)) * (cfg["m"] * cfg["k"] + cfg["k"] * cfg["n"])
        parallelism = f"batch split over {world} GPU(s), {batch // max(world, 1)} problems each"
    else:
        per_gpu = 4 * (cfg["m"] // gr * cfg["k"] + cfg["k"] * cfg["n"] // gc)
        parallelism = (f"{gr}x{gc} grid of row/column-band shards" if world > 1
                       else "single GPU")
    l2 = (f"inputs larger than L2 ({per_gpu / 2**30:.2f} GiB per GPU); no flush"
          if per_gpu >= (256 << 20) else
          "inputs smaller than L2: a 256 MiB buffer written before each timed step")
    return {"workload": cfg["workload"], "M": cfg["m"], "N": cfg["n"], "K": cfg["k"],
            "batch": batch, "depth": args.depth, "basis": args.basis, "layout": "row-major",
            "math": args.math, "l2": l2, "parallelism": parallelism}


# ---------------------------------------------------------------------------
# Clock sampling during the timed region.
# ---------------------------------------------------------------------------

class ClockSampler:
    """SM clock / throttle samples, each stamped with host time, in the CSV
    form of ``nvidia-smi --query-gpu=CLOCK_FIELDS``: NVML polled every 10 ms
    (nvidia-smi every 50 ms where NVML is missing).  summary() keeps the
    samples inside [window] (the timed region), else the nearest two."""

    REASON_BITS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
                   ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4))

    def __init__(self, device_index: int, pci_bus_id: str | None = None):
        self.device_index = device_index
        self.pci_bus_id = pci_bus_id
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self._thread = None
        self._stop = threading.Event()
        self.window: tuple[float, float] | None = None

    def __enter__(self):
        handle = self._nvml_handle()
        if handle is not None:
            self._thread = threading.Thread(target=self._poll_nvml, args=(handle,), daemon=True)
            self._thread.start()
            return self
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

    def _nvml_handle(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            if self.pci_bus_id:
                return pynvml.nvmlDeviceGetHandleByPciBusId(self.pci_bus_id)
            return pynvml.nvmlDeviceGetHandleByIndex(self.device_index)
        except Exception:
            return None

    def _poll_nvml(self, handle):
        import pynvml
        state = lambda on: "Active" if on else "Not Active"  # noqa: E731
        while not self._stop.is_set():
            try:
                sm = pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)
                mx = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
                pw = pynvml.nvmlDeviceGetPowerUsage(handle) / 1000.0
                rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                flags = ", ".join(state(rs & bit) for _, bit in self.REASON_BITS)
                self.lines.append((time.time(),
                                   f"{self.device_index}, {sm}, {mx}, {pw:.1f}, {rs:#x}, {flags}"))
            except Exception:
                pass
            self._stop.wait(0.01)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def __exit__(self, *exc):
        self._stop.set()
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
        names = [n for n, _ in self.REASON_BITS]
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
# every host core over a row-band sample of the workload.
# ---------------------------------------------------------------------------

def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


class all_host_threads:
    """BLAS and OpenMP pools at every host core for the block, whatever the
    launcher exported (torchrun sets OMP_NUM_THREADS=1 for N > 1)."""

    def __enter__(self):
        self.cores = host_cores()
        self._ctl = None
        try:
            from threadpoolctl import threadpool_limits
            self._ctl = threadpool_limits(limits=self.cores)
        except Exception:
            self._ctl = None
        return self

    def __exit__(self, *exc):
        if self._ctl is not None:
            self._ctl.restore_original_limits()

    def threads(self) -> int:
        try:
            from threadpoolctl import threadpool_info
            counts = [i.get("num_threads", 0) for i in threadpool_info()
                      if i.get("user_api") == "blas"]
            if counts:
                return int(max(counts))
        except Exception:
            pass
        return self.cores


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


def fp64_gemm_sample(a: np.ndarray, b: np.ndarray, units: int) -> tuple[float, float]:
    """The classical FP64 numpy GEMM (the error oracle) on the same sample."""
    if a.ndim == 3:
        aa = [a[i].astype(np.float64) for i in range(units)]
        bb = [b[i].astype(np.float64) for i in range(units)]
        t0 = time.perf_counter()
        for x, y in zip(aa, bb):
            x @ y
        dt = time.perf_counter() - t0
        return dt, 2.0 * units * a.shape[1] * a.shape[2] * b.shape[2]
    a64 = a[:units].astype(np.float64)
    b64 = b.astype(np.float64)
    t0 = time.perf_counter()
    a64 @ b64
    dt = time.perf_counter() - t0
    return dt, 2.0 * units * b.shape[0] * b.shape[1]


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


def _grow_sample(fn, units, top, target_s):
    dt, flops = fn(units)
    while dt < target_s / 3 and units * 2 <= top:
        units *= 2
        dt, flops = fn(units)
    return units, dt, flops


def cpu_baseline(a, b, depth, basis, target_s: float) -> dict:
    with all_host_threads() as pool:
        units, top = _sample_units(a, depth)
        units, dt, flops = _grow_sample(lambda u: cpu_sample(a, b, depth, basis, u), units, top,
                                        target_s)
        g_units, g_dt, g_flops = _grow_sample(lambda u: fp64_gemm_sample(a, b, u), units, top,
                                              target_s / 2)
        threads = pool.threads()
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": _describe_sample(a, b, units, depth, basis, dt),
            "fp64_classical_gemm": {
                "value": g_flops / g_dt / 1e12, "unit": "TFLOP/s", "cores": threads,
                "sample": f"numpy FP64 A@B on the first {g_units} "
                          f"{'problems' if a.ndim == 3 else 'rows of A'}: {g_dt:.2f} s"}}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    a, b = make_inputs(args.cfg)
    depth = args.depth
    with all_host_threads() as pool:
        units, top = _sample_units(a, depth)
        units, _, _ = _grow_sample(lambda u: cpu_sample(a, b, depth, args.basis, u), units, top,
                                   args.cpu_seconds)
        for _ in range(args.warmup):
            cpu_sample(a, b, depth, args.basis, units)
        times = []
        flops = 0.0
        for _ in range(args.steps):
            dt, flops = cpu_sample(a, b, depth, args.basis, units)
            times.append(dt)
        g_dt, g_flops = fp64_gemm_sample(a, b, units)
        threads = pool.threads()
    step = sum(times) / len(times)
    value = flops / step / 1e12
    base = {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": _describe_sample(a, b, units, depth, args.basis, step),
            "fp64_classical_gemm": {
                "value": g_flops / g_dt / 1e12, "unit": "TFLOP/s", "cores": threads,
                "sample": f"numpy FP64 A@B on the same {units} "
                          f"{'problems' if a.ndim == 3 else 'rows of A'}: {g_dt:.2f} s"}}
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": step * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": line_config(args, world),
            "reference_run": {"sample_units": units, "where": "host cores of rank 0, BLAS threads "
                              "set to every core whatever the launcher exported"},
            "cpu_baseline": base,
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Same-box comparators: cuBLAS SGEMM in the reference's mode, the reference's
# CUDA BAG (oracle/_ref, compiled from its headers; a checker here).
# ---------------------------------------------------------------------------

class Cublas:
    """cublasSgemm through ctypes on a given stream, in CUBLAS_PEDANTIC_MATH with
    atomics not allowed -- the reference baseline's mode
    (benchmarks/cuda/fp32_baseline.cu:199-202)."""

    def __init__(self, stream_ptr: int):
        import torch
        root = os.path.dirname(os.path.dirname(torch.__file__))
        cands = sorted(glob.glob(os.path.join(root, "nvidia", "cublas", "lib", "libcublas.so*")))
        self.lib = ctypes.CDLL(cands[0] if cands else "libcublas.so")
        self.h = ctypes.c_void_p()
        self._ok(self.lib.cublasCreate_v2(ctypes.byref(self.h)), "cublasCreate")
        self._ok(self.lib.cublasSetStream_v2(self.h, ctypes.c_void_p(stream_ptr)), "cublasSetStream")
        self._ok(self.lib.cublasSetMathMode(self.h, 2), "cublasSetMathMode(PEDANTIC)")
        self._ok(self.lib.cublasSetAtomicsMode(self.h, 0), "cublasSetAtomicsMode(NOT_ALLOWED)")
        ver = ctypes.c_int(0)
        self._ok(self.lib.cublasGetVersion_v2(self.h, ctypes.byref(ver)), "cublasGetVersion")
        self.version = ver.value
        self.alpha = ctypes.c_float(1.0)
        self.beta = ctypes.c_float(1.0)

    @staticmethod
    def _ok(status, what):
        if status != 0:
            raise RuntimeError(f"{what} failed with cuBLAS status {status}")

    def gemm(self, a, b, c):
        """Row-major c += a @ b (2-D or batched 3-D contiguous float32 tensors)."""
        vp = ctypes.c_void_p
        if a.ndim == 3:
            batch, m, k = a.shape
            n = b.shape[2]
            self._ok(self.lib.cublasSgemmStridedBatched(
                self.h, 0, 0, n, m, k, ctypes.byref(self.alpha), vp(b.data_ptr()), n,
                ctypes.c_longlong(k * n), vp(a.data_ptr()), k, ctypes.c_longlong(m * k),
                ctypes.byref(self.beta), vp(c.data_ptr()), n, ctypes.c_longlong(m * n), batch),
                "cublasSgemmStridedBatched")
        else:
            m, k = a.shape
            n = b.shape[1]
            self._ok(self.lib.cublasSgemm_v2(
                self.h, 0, 0, n, m, k, ctypes.byref(self.alpha), vp(b.data_ptr()), n,
                vp(a.data_ptr()), k, ctypes.byref(self.beta), vp(c.data_ptr()), n), "cublasSgemm")

    def close(self):
        if self.h:
            self.lib.cublasDestroy_v2(self.h)
            self.h = ctypes.c_void_p()


def reference_cuda():
    """The reference's CUDA BAG (bag_cuda::matmul, include/bag/cuda/bag.cuh:249-260),
    or None where oracle/_ref has not been built."""
    if not os.path.exists(REF_LIB):
        return None
    lib = ctypes.CDLL(REF_LIB)
    lib.ref_bag_matmul.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 5 + [ctypes.c_void_p]
    lib.ref_last_error.restype = ctypes.c_char_p
    return lib


def reference_step(ref, a, b, c, depth: int, basis: str, stream_ptr: int) -> None:
    """c += a @ b (row-major) through the reference's CUDA BAG: its column-major
    C^T = B^T A^T, ColumnTile8 backend, Batched schedule.  The reference takes
    square n x n matrices with ld = n only, so a batch is a loop of calls and a
    rectangular problem whose extents are multiples of the smallest, s, is
    composed from square s^3 calls on packed sub-blocks
    (C_il += sum_j A_ij B_jl)."""
    import torch
    basis_id = {"minimal": 0, "full": 1}[basis]

    def square(x, y, z, n):
        st = ref.ref_bag_matmul(y.data_ptr(), x.data_ptr(), z.data_ptr(), n, depth, basis_id, 2,
                                0, ctypes.c_void_p(stream_ptr))
        if st != 0:
            raise RuntimeError(ref.ref_last_error().decode())

    if a.ndim == 3:
        for i in range(a.shape[0]):
            square(a[i], b[i], c[i], a.shape[1])
        return
    m, k = a.shape
    n = b.shape[1]
    if m == k == n:
        square(a, b, c, m)
        return
    s = min(m, k, n)
    if m % s or k % s or n % s:
        raise RuntimeError("the reference takes square matrices only")
    for i in range(m // s):
        for col in range(n // s):
            block = torch.zeros(s, s, device=c.device) if n != s else c[i * s:(i + 1) * s]
            for j in range(k // s):
                square(a[i * s:(i + 1) * s, j * s:(j + 1) * s].contiguous(),
                       b[j * s:(j + 1) * s, col * s:(col + 1) * s].contiguous(), block, s)
            if n != s:
                c[i * s:(i + 1) * s, col * s:(col + 1) * s] += block


def frobenius_sums(a, b, outs, panel: int = 2048):
    """(sum of squared differences per C in `outs`, sum of squares of A@B)
    against an FP64 GEMM on the GPU, in column panels (a batch: per problem)."""
    num = [0.0] * len(outs)
    den = 0.0
    batched = a.ndim == 3
    for i in range(a.shape[0] if batched else 1):
        ai, bi = (a[i], b[i]) if batched else (a, b)
        a64 = ai.double()
        for j in range(0, bi.shape[1], panel):
            exact = a64 @ bi[:, j:j + panel].double()
            den += float((exact * exact).sum())
            for o, c in enumerate(outs):
                ci = c[i] if batched else c
                d = ci[:, j:j + panel].double() - exact
                num[o] += float((d * d).sum())
        del a64
    return num, den


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
    row_group = col_group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    torch.backends.cuda.matmul.allow_tf32 = False
    bag.set_math_mode(args.math)

    cfg, depth = args.cfg, args.depth
    M, N, K, batch = cfg["m"], cfg["n"], cfg["k"], cfg["batch"]
    gr, gc = shard_grid(world)
    config = line_config(args, world)
    a_np, b_np = make_inputs(cfg)
    pieces = None
    if batch > 1:
        # A batch: every rank takes batch/world whole problems.
        if batch % world:
            raise SystemExit("the batch must split evenly over the GPUs")
        nb = batch // world
        a_shard = np.ascontiguousarray(a_np[rank * nb:(rank + 1) * nb])
        b_shard = np.ascontiguousarray(b_np[rank * nb:(rank + 1) * nb])
        mg, ng = M, N
    else:
        if M % ((4 << depth) * gr) or N % ((4 << depth) * gc):
            raise SystemExit("the problem must split into aligned bands for this GPU count")
        nb = 1
        rows = band_rows(M, depth, gr, rank // gc)
        cols = band_rows(N, depth, gc, rank % gc)
        mg, ng = rows.size, cols.size
        a_shard = np.ascontiguousarray(a_np[rows]) if gr > 1 else a_np
        b_shard = np.ascontiguousarray(b_np[:, cols]) if gc > 1 else b_np
        if world > 1:
            pieces = upload_pieces(mg, K, gr, gc, rank)
    if world > 1:
        # Every rank creates every group, in the same order (NCCL communicators
        # for the e2e all-gathers).
        rgs = [dist.new_group([i * gc + j for j in range(gc)]) for i in range(gr)]
        cgs = [dist.new_group([i * gc + j for i in range(gr)]) for j in range(gc)]
        row_group, col_group = rgs[rank // gc], cgs[rank % gc]
    keep_full = rank == 0   # rank 0 checks the reference's error on the full problem
    if not keep_full:
        del a_np, b_np
    lead = (nb,) if batch > 1 else ()

    # Device buffers (the `value` inputs, resident).
    a_dev = torch.from_numpy(a_shard).to(device)
    b_dev = torch.from_numpy(b_shard).to(device)
    c_dev = torch.zeros(lead + (mg, ng), dtype=torch.float32, device=device)
    # Row-major C(mg x ng) = A B is the column-major ng x mg problem.
    ws = bag.Workspace.for_problem(ng, mg, K, depth, args.basis, batch=nb)
    stream = torch.cuda.current_stream()
    gemm = bag.sgemm_batched if batch > 1 else bag.sgemm

    def step():
        gemm(a_dev, b_dev, c_dev, beta=1.0, depth=depth, basis=args.basis, workspace=ws)

    def barrier():
        if world > 1:
            dist.barrier()

    def reduce(x: float, op) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=op)
        return float(t.item())

    reduce_max = lambda x: reduce(x, dist.ReduceOp.MAX if world > 1 else None)  # noqa: E731
    reduce_sum = lambda x: reduce(x, dist.ReduceOp.SUM if world > 1 else None)  # noqa: E731

    def per_rank(x: float) -> list[float]:
        if world == 1:
            return [x]
        t = torch.zeros(world, dtype=torch.float64, device=device)
        t[rank] = x
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return [float(v) for v in t.tolist()]

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

    w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    step()
    torch.cuda.synchronize()
    w0.record()
    for _ in range(args.warmup):
        step()
    w1.record()
    torch.cuda.synchronize()
    warm_ms = w0.elapsed_time(w1) / args.warmup
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
    props = torch.cuda.get_device_properties(device)
    pci = None
    if hasattr(props, "pci_bus_id"):
        pci = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    soak_steps = max(1, int(SOAK_S * 1e3 / max(warm_ms, 1e-3)) + 1)
    with ClockSampler(local, pci) as clocks:
        # Untimed soak: at every N the timed region starts after >= 1 s of
        # load, at the power-steady clock.
        for _ in range(soak_steps):
            step()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        launches0 = bag.launch_count()
        host0 = time.time()
        t_start.record()
        for i in range(args.steps):
            # The library's profiling hooks are set before the step's start
            # event: with a flush between steps, the step's events time the
            # call alone.
            if flush is not None:
                flush.fill_(float(i))
            bag.profile_events(*pairs[i])
            bag.profile_phase_events(phases[i][1], phases[i][2])
            if flush is not None:
                step_events[i][0].record()
            phases[i][0].record()
            step()
            if flush is not None:
                step_events[i][1].record()
        bag.profile_events(None, None)
        bag.profile_phase_events(None, None)
        t_end.record()
        torch.cuda.synchronize()
        clocks.window = (host0, time.time())
        time.sleep(0.05)
    barrier()
    launches = reduce_sum(bag.launch_count() - launches0)
    leaf_path = bag.last_leaf_path()
    leaf_kernel = bag.last_leaf_kernel()
    if flush is not None:
        ms = reduce_max(sum(s0.elapsed_time(s1) for s0, s1 in step_events)) / args.steps
    else:
        ms = reduce_max(t_start.elapsed_time(t_end)) / args.steps
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
    sms = props.multi_processor_count
    csum = clocks.summary()
    max_mhz = csum["sm_max_mhz"] or 1965.0
    nominal = sms * 128 * 2 * max_mhz * 1e6 / 1e12
    sink = torch.empty(sms * 1024, dtype=torch.float32, device=device)
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
    del sink

    # End to end through the public API, host buffers in and out, pipelined
    # like a serving loop: step i+1's inputs are uploaded on one copy stream
    # (and, on N GPUs, all-gathered on a communication stream) while step i
    # computes, and step i's C is read back on another stream while step i+1
    # computes (two buffer sets).  Every step moves its own inputs from host
    # memory and its result back, each host byte once across all ranks.
    comp = torch.cuda.current_stream()
    h2d_s, d2h_s = torch.cuda.Stream(device), torch.cuda.Stream(device)
    h2d_b = torch.cuda.Stream(device)   # B's upload on its own copy stream, beside A's
    comm_s = torch.cuda.Stream(device)
    if pieces is not None:
        a_up = np.ascontiguousarray(a_shard[pieces["a_rows"][0]:pieces["a_rows"][1]])
        b_up = np.ascontiguousarray(b_shard[pieces["b_rows"][0]:pieces["b_rows"][1]])
    else:
        a_up, b_up = a_shard, b_shard
    a_host = torch.from_numpy(a_up).pin_memory()
    b_host = torch.from_numpy(b_up).pin_memory()
    del a_up, b_up
    c_host = [torch.empty(lead + (mg, ng), dtype=torch.float32).pin_memory() for _ in range(2)]
    a2 = [a_dev, torch.empty_like(a_dev)]
    b2 = [b_dev, torch.empty_like(b_dev)]
    c2 = [c_dev, torch.empty_like(c_dev)]
    if pieces is not None:
        ap = [torch.empty(tuple(a_host.shape), dtype=torch.float32, device=device) for _ in range(2)]
        bp = [torch.empty(tuple(b_host.shape), dtype=torch.float32, device=device) for _ in range(2)]
    up_done = [torch.cuda.Event(), torch.cuda.Event()]
    up_b_done = [torch.cuda.Event(), torch.cuda.Event()]
    gath_done = [torch.cuda.Event(), torch.cuda.Event()]
    comp_done = [torch.cuda.Event(), torch.cuda.Event()]
    down_done = [torch.cuda.Event(), torch.cuda.Event()]
    e2e_steps = max(args.steps, 20)
    gath_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(e2e_steps)]

    def e2e_run(steps: int, start_event=None, timed=False) -> int:
        if start_event is not None:
            h2d_s.wait_event(start_event)
        for i in range(steps):
            sl = i % 2
            # A and B go up on two copy streams at once: one copy stream alone
            # left part of the host-to-device bandwidth unused (measured on
            # B200: e2e 186.5 -> 200.4 TFLOP/s at cfg3; four streams, 188.8).
            # B's stream first waits on the work already queued on A's (the
            # start event, the previous step's uploads).
            reuse = comp_done[sl] if pieces is None else gath_done[sl]
            with torch.cuda.stream(h2d_b):
                h2d_b.wait_stream(h2d_s)
                if i >= 2:
                    h2d_b.wait_event(reuse)   # step i-2 no longer reads slot sl
                (b2 if pieces is None else bp)[sl].copy_(b_host, non_blocking=True)
                up_b_done[sl].record(h2d_b)
            with torch.cuda.stream(h2d_s):
                if i >= 2:
                    h2d_s.wait_event(reuse)
                (a2 if pieces is None else ap)[sl].copy_(a_host, non_blocking=True)
                h2d_s.wait_event(up_b_done[sl])
                up_done[sl].record(h2d_s)
            if pieces is not None:
                with torch.cuda.stream(comm_s):
                    comm_s.wait_event(up_done[sl])
                    if i >= 2:
                        comm_s.wait_event(comp_done[sl])  # step i-2's gemm read the shards
                    if timed:
                        gath_ev[i][0].record(comm_s)
                    dist.all_gather_into_tensor(a2[sl], ap[sl], group=row_group)
                    dist.all_gather_into_tensor(b2[sl], bp[sl], group=col_group)
                    if timed:
                        gath_ev[i][1].record(comm_s)
                    gath_done[sl].record(comm_s)
                comp.wait_event(gath_done[sl])
            else:
                comp.wait_event(up_done[sl])
            if i >= 2:
                comp.wait_event(down_done[sl])        # step i-2's C has been read back
            gemm(a2[sl], b2[sl], c2[sl], beta=0.0, depth=depth, basis=args.basis, workspace=ws)
            comp_done[sl].record(comp)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(comp_done[sl])
                c_host[sl].copy_(c2[sl], non_blocking=True)
                down_done[sl].record(d2h_s)
        comp.wait_stream(h2d_s)
        comp.wait_stream(h2d_b)
        comp.wait_stream(d2h_s)
        comp.wait_stream(comm_s)
        return (steps - 1) % 2

    # The timed run starts and ends with an empty pipeline (the first upload
    # and the last read-back overlap nothing), so it runs at least 20 steps to
    # report a serving loop's steady rate.
    e2e_run(2)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    last = e2e_run(e2e_steps, start_event=e0, timed=True)
    e1.record(comp)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = reduce_max(e0.elapsed_time(e1)) / e2e_steps
    gather_ms = per_rank(sum(s.elapsed_time(e) for s, e in gath_ev) / e2e_steps
                         if pieces is not None else 0.0)
    c_res = c2[last]   # this run's final C = A@B, for the accuracy check
    up_bytes = 4.0 * (a_host.numel() + b_host.numel())
    h2d = int(reduce_sum(up_bytes))                 # every rank's uploads
    d2h = int(reduce_sum(4.0 * c_res.numel()))      # every rank's C shard
    del c_host, a_host, b_host
    if pieces is not None:
        del ap, bp
    del a2[1], b2[1], c2[1 - last]
    torch.cuda.empty_cache()

    # Comparators on one GPU: cuBLAS SGEMM (torch default math, and cuBLAS in
    # the reference's PEDANTIC mode through ctypes), this library's FFMA
    # path, and the reference's CUDA BAG, on the same inputs.
    comparators = {}
    c_ffma = None
    if rank == 0 and world == 1 and not args.no_comparators:
        def timed(fn, reps):
            fn()
            torch.cuda.synchronize()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            for _ in range(reps):
                fn()
            t1.record()
            torch.cuda.synchronize()
            return t0.elapsed_time(t1) / reps

        reps = min(args.steps, 5)
        c_tmp = torch.zeros_like(c_res)
        if leaf_path != "ffma":
            bag.set_math_mode("ffma")
            fms = timed(lambda: gemm(a_dev, b_dev, c_tmp, beta=1.0, depth=depth, basis=args.basis,
                                     workspace=ws), reps)
            bag.set_math_mode(args.math)
            comparators["bag_ffma_path"] = {"tflops": flops_total / (fms * 1e-3) / 1e12,
                                            "ms_per_step": fms,
                                            "how": "same call, bag_set_math_mode(BAG_MATH_FFMA)"}
        cms = timed(lambda: c_tmp.baddbmm_(a_dev, b_dev) if batch > 1 else c_tmp.addmm_(a_dev, b_dev),
                    reps)
        comparators["cublas_sgemm_fp32"] = {"tflops": flops_total / (cms * 1e-3) / 1e12,
                                            "ms_per_step": cms,
                                            "how": "torch addmm_/baddbmm_, allow_tf32=False "
                                                   "(cuBLAS FP32, default math)"}
        try:
            cb = Cublas(stream.cuda_stream)
            pms = timed(lambda: cb.gemm(a_dev, b_dev, c_tmp), reps)
            comparators["cublas_sgemm_pedantic"] = {
                "tflops": flops_total / (pms * 1e-3) / 1e12, "ms_per_step": pms,
                "cublas_version": cb.version,
                "how": "cublasSgemm(StridedBatched) via ctypes, CUBLAS_PEDANTIC_MATH, atomics not "
                       "allowed (the reference baseline's mode, fp32_baseline.cu:199-202)"}
            cb.close()
        except Exception as exc:   # reported, not fatal
            comparators["cublas_sgemm_pedantic"] = {"error": str(exc)[:200]}
        del c_tmp
        if leaf_path != "ffma":
            bag.set_math_mode("ffma")
            c_ffma = torch.zeros_like(c_res)
            gemm(a_dev, b_dev, c_ffma, beta=0.0, depth=depth, basis=args.basis, workspace=ws)
            bag.set_math_mode(args.math)
    del ws
    torch.cuda.empty_cache()

    # Accuracy at every N: each rank's C shard against an FP64 GEMM of its own
    # A and B shards on its GPU; the sums add up over ranks to the full C's
    # relative Frobenius error.  Rank 0 also runs the reference's CUDA BAG on
    # the full inputs (3 fresh runs, median) for the bound's base, and at
    # N = 1 times it beside the comparators.
    outs = [c_res] + ([c_ffma] if c_ffma is not None else [])
    num, den = frobenius_sums(a_dev, b_dev, outs)
    num0, den_all = reduce_sum(num[0]), reduce_sum(den)
    accuracy = {"rel_frobenius_vs_fp64": (num0 / den_all) ** 0.5,
                "how": "every rank's C shard vs an FP64 GEMM of its shards (GPU), sums "
                       "all-reduced over ranks"}
    if c_ffma is not None:
        accuracy["ffma_path_rel_frobenius_vs_fp64"] = (num[1] / den) ** 0.5
    del outs, c_ffma
    ref_info = None
    if rank == 0:
        ref = reference_cuda()
        if ref is not None and args.basis in ("minimal", "full"):
            del a_dev, b_dev, c_dev, c_res, c2
            torch.cuda.empty_cache()
            fa = torch.from_numpy(a_np).to(device)
            fb = torch.from_numpy(b_np).to(device)
            errs, refs = [], []
            try:
                for _ in range(3):
                    cr = torch.zeros(fa.shape[:-1] + (fb.shape[-1],), device=device)
                    reference_step(ref, fa, fb, cr, depth, args.basis, stream.cuda_stream)
                    refs.append(cr)
                torch.cuda.synchronize()
                rnum, rden = frobenius_sums(fa, fb, refs)
                errs = [(x / rden) ** 0.5 for x in rnum]
                del refs
                ref_info = {"reference_cuda_rel_frobenius": float(np.median(errs)),
                            "reference_cuda_rel_frobenius_runs": errs}
                if world == 1 and not args.no_comparators:
                    cr = torch.zeros(fa.shape[:-1] + (fb.shape[-1],), device=device)
                    fn = lambda: reference_step(ref, fa, fb, cr, depth, args.basis,  # noqa: E731
                                                stream.cuda_stream)
                    fn()
                    torch.cuda.synchronize()
                    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    reps = 3
                    r0.record()
                    for _ in range(reps):
                        fn()
                    r1.record()
                    torch.cuda.synchronize()
                    rms = r0.elapsed_time(r1) / reps
                    comparators["reference_cuda_bag"] = {
                        "tflops": flops_total / (rms * 1e-3) / 1e12, "ms_per_step": rms,
                        "rel_frobenius_vs_fp64": ref_info["reference_cuda_rel_frobenius"],
                        "how": "the reference's bag_cuda::matmul (ColumnTile8, Batched, "
                               "include/bag/cuda/bag.cuh:249-260) compiled unmodified from its "
                               "headers into oracle/_ref; C^T = B^T A^T for row-major; a loop "
                               "of 64 calls for a batch"}
                    del cr
            except Exception as exc:
                ref_info = {"reference_cuda_error": str(exc)[:200]}
            del fa, fb
            torch.cuda.empty_cache()
    if rank == 0:
        err = accuracy["rel_frobenius_vs_fp64"]
        if ref_info and "reference_cuda_rel_frobenius" in ref_info:
            accuracy.update(ref_info)
            r = ref_info["reference_cuda_rel_frobenius"]
            accuracy.update({"ratio_to_reference": err / r,
                             "bound": "<= 1.25x the reference CUDA BAG's rel-F (median of 3 runs, "
                                      "same inputs, same depth) and <= 1e-4",
                             "within_bound": err <= min(1.25 * r, 1e-4)})
        elif "ffma_path_rel_frobenius_vs_fp64" in accuracy:
            if ref_info:
                accuracy.update(ref_info)
            f = accuracy["ffma_path_rel_frobenius_vs_fp64"]
            accuracy.update({"bound": "<= 1.25x the FFMA path (the reference's sequential fmaf "
                                      "numerics; reference CUDA BAG unavailable) and <= 1e-4",
                             "within_bound": err <= min(1.25 * f, 1e-4)})
        else:
            accuracy.update({"bound": "<= 1e-4", "within_bound": err <= 1e-4})

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(a_np, b_np, depth, args.basis, args.cpu_seconds)

    # End to end from GPU 0 through the one-process multi-GPU entry point.
    multi = None
    if world > 1:
        multi = e2e_from_gpu0(args, bag, dist, torch, rank, world, a_np if rank == 0 else None,
                              b_np if rank == 0 else None)

    if rank == 0:
        if leaf_path == "3xtf32":
            peaks = measured_peaks()
            tf32 = peaks.get("bf16_tflops", 1590.0) / 2.0
            sustained = peaks.get("bf16_tflops_sustained", 1400.0) / 2.0
            # The workspace was created in 3xTF32 mode, so the call runs the
            # prepare pass (prep_tree_kernel), the leaf kernel on the prepared
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
            # The leaf launches are timed inside a long step (a >= 1 s soak, then
            # the timed steps), so the denominator is the sustained figure; the
            # burst one is reported beside it.
            roofline = {"bound": "tensor", "kernel": kname,
                        "achieved": leaf_tflops, "peak": sustained / 3.0, "unit": "TFLOP/s",
                        "frac": leaf_tflops / (sustained / 3.0),
                        "traffic": traffic_for(args, world, kfile),
                        "prepare_and_materialise_ms": ms - leaf_ms,
                        "peak_source": "MEASURED_PEAKS.json bf16_tflops_sustained (of measured; "
                                       "the kernel runs inside a long power-capped step) / 2 "
                                       "(dense TF32 = half the bf16 rate) / 3 (three MMAs per "
                                       "leaf product: hi*hi, hi*lo, lo*hi)",
                        "peak_burst": tf32 / 3.0,
                        "frac_of_burst": leaf_tflops / (tf32 / 3.0),
                        "leaf_ms": leaf_ms, "algorithmic_flops_per_launch": f_exec}
        else:
            roofline = {"bound": "compute", "kernel": "leaf_ws_kernel / leaf_gemm_kernel "
                                                      "(FP32 FFMA SIMT)",
                        "achieved": leaf_tflops, "peak": nominal, "unit": "TFLOP/s",
                        "frac": leaf_tflops / nominal,
                        "traffic": traffic_for(args, world, "leaf_gemm_cfg3_traffic.txt"),
                        "peak_source": f"nominal FP32 FFMA {sms} SM x 128 lanes x 2 x "
                                       f"{max_mhz:.0f} MHz (MEASURED_PEAKS.json has no FP32 "
                                       f"SIMT figure)",
                        "ffma_probe_tflops": probe, "frac_of_probe": leaf_tflops / probe,
                        "leaf_ms": leaf_ms, "algorithmic_flops_per_launch": f_exec}
        e2e = {"value": flops_total / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
               "steps": e2e_steps,
               "how": "public sgemm API from pinned host buffers; uploads (A and B on two copy "
                      "streams; on N GPUs followed by NCCL all-gathers) of step i+1 and the "
                      "read-back of step i overlap step i's compute (2 buffer sets); every host "
                      "byte crosses PCIe once"}
        if world > 1:
            e2e["allgather_ms_per_step_by_rank"] = gather_ms
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": config, "leaf_math": leaf_path,
            "e2e": e2e,
            "roofline": roofline,
            "ffma_probe_tflops": probe,
            "clocks": {k: csum[k] for k in ("sm_mhz", "sm_max_mhz", "reasons",
                                            "samples_in_timed_region")},
            "soak": {"steps": soak_steps, "seconds_target": SOAK_S},
            "gpu_launches": int(launches),
            "phases_ms": phases_ms,
            "executed_tflops": f_exec * world / (ms * 1e-3) / 1e12,
            "accuracy": accuracy,
        }
        if multi is not None:
            line["e2e_from_gpu0"] = multi
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if comparators:
            line["comparators"] = comparators
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def e2e_from_gpu0(args, bag, dist, torch, rank, world, a_np, b_np):
    """Rank 0 times ``bag_sgemm_multi`` with A, B and C on GPU 0 over GPUs
    0..N-1 (peer copies of the shards, compute, C bands copied back) after the
    other ranks have freed their buffers; they wait on the host (the process
    group's store), launching nothing, until it is done."""
    from datetime import timedelta
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    dist.barrier()
    store = None
    try:
        store = dist.distributed_c10d._get_default_store()
    except Exception:
        store = None
    if store is None:
        return {"error": "no process-group store to wait on"} if rank == 0 else None
    key = "bag_b200_e2e_from_gpu0_done"
    if rank != 0:
        store.wait([key], timedelta(seconds=900))
        return None
    result = None
    try:
        if args.cfg["batch"] > 1:
            result = {"skipped": "batched configs split whole problems; sgemm_multi takes one"}
            return result
        m, k = a_np.shape
        n = b_np.shape[1]
        dev0 = torch.device("cuda", 0)
        a = torch.from_numpy(a_np).to(dev0)
        b = torch.from_numpy(b_np).to(dev0)
        c = torch.zeros(m, n, device=dev0)
        mws = bag.MultiWorkspace(list(range(world)), m, n, k, depth=args.depth, basis=args.basis)
        s = torch.cuda.current_stream(dev0)
        bag.sgemm_multi(a, b, c, mws, beta=0.0, stream=s)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        e0.record(s)
        for _ in range(reps):
            bag.sgemm_multi(a, b, c, mws, beta=0.0, stream=s)
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        num, den = frobenius_sums(a, b, [c])
        result = {"value": 2.0 * m * n * k / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                  "ms_per_step": ms, "steps": reps, "devices": world,
                  "rel_frobenius_vs_fp64": (num[0] / den) ** 0.5,
                  "how": "bag_sgemm_multi from one process: A, B, C on GPU 0; shards by peer "
                         "copies over NVLink, C bands copied back; CUDA events on GPU 0's stream"}
        del mws, a, b, c
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    except Exception as exc:   # reported, not fatal
        result = {"error": str(exc)[:300]}
    finally:
        store.set(key, "1")
    return result


def measured_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def traffic_for(args, world: int, name: str):
    """The committed ncu traffic figure, which is per cfg3 leaf launch on one
    GPU: reported for that workload only (null for the other configs and for
    a rank's shard at N > 1, whose launches are smaller)."""
    if getattr(args, "config", "cfg3") != "cfg3" or world != 1 or args.depth != 2:
        return None
    return read_traffic(name)


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
