"""Effective TFLOP/s of one GEMM shape at each BAG depth, to tune the depth.

``python -m bag_b200.depth_sweep --math 3xtf32 --shapes 4096,16384,8192x4096x16384``
prints one JSON line per shape: 2MNK/t for each depth the shape allows, and
the leaf kernel each depth ran.  Every depth is timed after a soak of
``--soak`` seconds of back-to-back calls, so a power-capped GPU is measured at
its steady clock, with CUDA events around ``--reps`` calls.  This is the
measurement behind ``BAG_DEPTH_AUTO``'s policy; run it on another GPU model to
re-check that policy there.
"""

from __future__ import annotations

import argparse
import json
import time


def parse_shape(text: str) -> tuple[int, int, int]:
    """"N" (square) or "MxNxK" (row-major C(M x N) = A(M x K) B(K x N))."""
    parts = [int(p) for p in text.lower().split("x")]
    if len(parts) == 1:
        parts = parts * 3
    if len(parts) != 3 or min(parts) <= 0:
        raise ValueError(f"shape {text!r} is not N or MxNxK with positive extents")
    return parts[0], parts[1], parts[2]


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--shapes", default="2048,4096,8192,16384",
                   help="comma-separated N or MxNxK")
    p.add_argument("--depths", default="0,1,2,3")
    p.add_argument("--basis", default="minimal")
    p.add_argument("--math", choices=("ffma", "3xtf32"), default="3xtf32")
    p.add_argument("--min-block", type=int, default=512,
                   help="skip depths whose blocks would be smaller than this")
    p.add_argument("--soak", type=float, default=0.6)
    p.add_argument("--reps", type=int, default=8)
    args = p.parse_args(argv)
    args.shapes = [parse_shape(s) for s in args.shapes.split(",") if s]
    args.depths = [int(d) for d in args.depths.split(",") if d]
    return args


def sweep_shape(bag, torch, m: int, n: int, k: int, args) -> dict:
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(m, k, device="cuda", generator=g)
    b = torch.randn(k, n, device="cuda", generator=g)
    c = torch.zeros(m, n, device="cuda")
    out = {"m": m, "n": n, "k": k, "math": args.math, "basis": args.basis, "tflops": {},
           "leaf_kernel": {}}
    for depth in args.depths:
        if min(m, n, k) >> depth < args.min_block:
            continue
        ws = bag.Workspace.for_problem(n, m, k, depth, args.basis)

        def call():
            bag.sgemm(a, b, c, beta=0.0, depth=depth, basis=args.basis, workspace=ws)

        call()
        torch.cuda.synchronize()
        t0 = time.time()
        while time.time() - t0 < args.soak:
            call()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.reps):
            call()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.reps
        out["tflops"][str(depth)] = round(2.0 * m * n * k / (ms * 1e-3) / 1e12, 1)
        out["leaf_kernel"][str(depth)] = bag.last_leaf_kernel()
        del ws
        torch.cuda.empty_cache()
    return out


def main(argv=None) -> None:
    args = parse_args(argv)
    import torch

    import bag_b200 as bag
    if not torch.cuda.is_available():
        raise SystemExit("depth_sweep needs a CUDA device")
    torch.backends.cuda.matmul.allow_tf32 = False
    bag.set_math_mode(args.math)
    for m, n, k in args.shapes:
        print(json.dumps(sweep_shape(bag, torch, m, n, k, args)), flush=True)


if __name__ == "__main__":
    main()
