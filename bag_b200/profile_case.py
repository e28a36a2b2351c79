"""Profiling and tile-sweep driver for the BAG kernels.

    python -m bag_b200.profile_case --n 4096 --depth 1          # one small case for ncu
    python -m bag_b200.profile_case --sweep                      # time the current tile config
    python -m bag_b200.profile_case --math 3xtf32 ...            # tensor-core leaf variant
    python -m bag_b200.profile_case --math 3xtf32 --fused ...    # ... without prepared operands
    python -m bag_b200.profile_case --devices 0,1 --n 16384 --depth 2 --math 3xtf32
                                                                 # time sgemm_multi

The case mode builds N(0,1) FP32 operands on cuda:0 (torch generator, seed 0)
and calls ``bag_b200.sgemm`` ``--calls`` times, so an ``ncu -k regex:leaf_gemm
-c 1`` capture sees the first leaf launch.  The sweep mode prints one JSON line
with effective and leaf-kernel TFLOP/s for a plain GEMM (depth 0, N=8192),
BAG depth 1 (N=8192) and BAG depth 2 (N=16384); the tile configuration is
the library default or the one pinned by ``BAG_B200_TILE``.
"""

from __future__ import annotations

import argparse
import json
import os


def _operands(n: int, depth: int, basis: str, fused: bool = False):
    import torch

    import bag_b200 as bag
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(n, n, device="cuda", generator=g)
    b = torch.randn(n, n, device="cuda", generator=g)
    c = torch.zeros(n, n, device="cuda")
    # In 3xTF32 mode a workspace (created in that mode) also holds the prepared
    # TF32 hi/lo leaf operands, so every depth gets one there.  `fused` sizes
    # the workspace as in FFMA mode instead (no prepared region): the
    # 3xTF32 calls then run the fused-prologue tensor kernel.
    mode = bag.get_math_mode()
    need_ws = depth >= 2 or basis != "minimal" or (mode == "3xtf32" and not fused)
    ws = None
    if need_ws:
        if fused:
            bag.set_math_mode("ffma")
        try:
            ws = bag.Workspace.for_problem(n, n, n, depth, basis)
        finally:
            bag.set_math_mode(mode)
    return a, b, c, ws


def run_case(n: int, depth: int, basis: str, calls: int, fused: bool = False) -> None:
    import torch

    import bag_b200 as bag
    a, b, c, ws = _operands(n, depth, basis, fused)
    for _ in range(calls):
        bag.sgemm(a, b, c, depth=depth, basis=basis, workspace=ws)
    torch.cuda.synchronize()
    print(f"ok n={n} depth={depth} basis={basis} calls={calls} "
          f"leaf_kernel={bag.last_leaf_kernel()}")


def run_sweep(reps: int = 3) -> dict:
    import torch

    import bag_b200 as bag
    out = {"tile": os.environ.get("BAG_B200_TILE", "default")}
    for name, n, depth in (("gemm8192_d0", 8192, 0), ("bag8192_d1", 8192, 1),
                           ("bag16384_d2", 16384, 2)):
        a, b, c, ws = _operands(n, depth, "minimal")
        for _ in range(2):
            bag.sgemm(a, b, c, depth=depth, workspace=ws)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(reps)]
        for s, e in evs:
            s.record()
            e.record()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for i in range(reps):
            bag.profile_events(*evs[i])
            bag.sgemm(a, b, c, depth=depth, workspace=ws)
        bag.profile_events(None, None)
        t1.record()
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1) / reps
        leaf = sum(s.elapsed_time(e) for s, e in evs) / reps
        fexec = 7 ** depth * 2.0 * (n / 2 ** depth) ** 3
        out[name] = {"ms": round(ms, 3), "eff_tflops": round(2.0 * n ** 3 / ms / 1e9, 2),
                     "leaf_ms": round(leaf, 3), "leaf_tflops": round(fexec / leaf / 1e9, 2)}
        del a, b, c, ws
        torch.cuda.empty_cache()
    return out


def run_multi(devices: list[int], n: int, depth: int, basis: str, calls: int) -> dict:
    """Time ``sgemm_multi`` over ``devices`` (inputs and output on the first):
    CUDA events on the first device's stream around ``calls`` calls after a
    warm-up; the single-device call on the same inputs beside it."""
    import torch

    import bag_b200 as bag
    torch.cuda.set_device(devices[0])
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(n, n, device="cuda", generator=g)
    b = torch.randn(n, n, device="cuda", generator=g)
    c = torch.zeros(n, n, device="cuda")

    def timed(fn) -> float:
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(calls):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / calls

    mws = bag.MultiWorkspace(devices, n, n, n, depth=depth, basis=basis)
    ms_multi = timed(lambda: bag.sgemm_multi(a, b, c, mws, beta=0.0))
    del mws
    ws = bag.Workspace.for_problem(n, n, n, depth, basis)
    ms_one = timed(lambda: bag.sgemm(a, b, c, beta=0.0, depth=depth, basis=basis, workspace=ws))
    flops = 2.0 * n ** 3
    return {"devices": devices, "grid": bag.multi_grid(len(devices)), "n": n, "depth": depth,
            "math": bag.get_math_mode(), "multi_ms": round(ms_multi, 3),
            "multi_tflops": round(flops / ms_multi / 1e9, 1), "one_gpu_ms": round(ms_one, 3),
            "one_gpu_tflops": round(flops / ms_one / 1e9, 1), "device_error": bag.device_error()}


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--n", type=int, default=4096)
    p.add_argument("--depth", type=int, default=1)
    p.add_argument("--basis", default="minimal")
    p.add_argument("--calls", type=int, default=3)
    p.add_argument("--sweep", action="store_true")
    p.add_argument("--math", default="ffma", choices=("ffma", "3xtf32"))
    p.add_argument("--devices", default=None, help="comma-separated: time sgemm_multi over them")
    p.add_argument("--fused", action="store_true",
                   help="3xtf32 without the prepared region: the fused-prologue tensor kernel")
    args = p.parse_args()
    import bag_b200 as bag
    bag.set_math_mode(args.math)
    if args.devices:
        devs = [int(x) for x in args.devices.split(",")]
        print(json.dumps(run_multi(devs, args.n, args.depth, args.basis, args.calls)), flush=True)
    elif args.sweep:
        print(json.dumps(run_sweep()), flush=True)
    else:
        run_case(args.n, args.depth, args.basis, args.calls, args.fused)


if __name__ == "__main__":
    main()
