#!/usr/bin/env python3
"""Generate golden fixtures from the reference's own Triton BAG code.

Runs ``bag_triton.bag_matmul`` and ``bag_triton.bag_primitive`` from the
reference checkout (``src/bag_triton``) under ``TRITON_INTERPRET=1`` on CPU
and writes their outputs, with the seeded inputs, to ``tests/golden/*.npz``.
The reference rejects non-CUDA tensors (``bag.py:998-999``,
``primitive.py:316-317``), so every tensor it sees, workspace included, is a
``torch.Tensor`` subclass whose ``is_cuda`` reports True; the reference files
are not modified.

Usage: python tests/golden/make_golden.py --reference <bag checkout> [--only cfg1]
(or set BAG_REFERENCE_ROOT instead of --reference).

``cfg1_triton_bag_n512.npz`` is BASELINE config 1 on its exact inputs:
A then B drawn U[-1,1) from ``numpy.random.default_rng(0)`` (``bench.make_inputs``),
512 x 512 row-major, one BAG level, the reference's default schedule ("auto",
grouped at this size); it stores the output and the first 64 draws of A and B,
so a test can check that it regenerates the same inputs.

This script needs the reference checkout and is run only where it exists;
the fixtures it writes are what travels.
"""

from __future__ import annotations

import argparse
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# Sizes follow tests/triton/test_bag.py:186 (2, 6, 64) plus two powers of two
# that exercise both Triton schedules on non-trivial tiles.
BAG_CASES = [
    # (name, n, layout, schedule, seed, dist)
    ("bag_n2_row_serial", 2, "row", "serial", 101, "half"),
    ("bag_n6_row_serial", 6, "row", "serial", 102, "half"),
    ("bag_n64_row_serial", 64, "row", "serial", 103, "half"),
    ("bag_n64_col_grouped", 64, "col", "grouped", 104, "half"),
    ("bag_n128_row_grouped", 128, "row", "grouped", 105, "pm1"),
    ("bag_n128_col_serial", 128, "col", "serial", 106, "pm1"),
    ("bag_n256_row_serial", 256, "row", "serial", 107, "normal"),
]

# Shapes and coefficients from tests/triton/test_primitive.py:141-150
# (the 511x509x513 case is left out to keep fixtures small).
PRIMITIVE_CASES = [
    ((1, 1, 1), (0, 0, 2, 0)),
    ((37, 29, 21), (1, -1, 1, -1)),
    ((63, 97, 35), (-1, 1, -2, 2)),
    ((257, 65, 33), (0, 1, 1, 1)),
    ((257, 64, 33), (-1, -1, 1, 1)),
    ((64, 257, 33), (-1, -1, 1, 1)),
    ((96, 80, 0), (0, 0, 2, -2)),
]


def _inputs(rng, shape, dist):
    if dist == "half":
        return rng.uniform(-0.5, 0.5, shape).astype(np.float32)
    if dist == "pm1":
        return rng.uniform(-1.0, 1.0, shape).astype(np.float32)
    return rng.standard_normal(shape, dtype=np.float32)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("BAG_REFERENCE_ROOT"),
                        help="root of the reference checkout (default: $BAG_REFERENCE_ROOT)")
    parser.add_argument("--only", choices=["cfg1"], default=None,
                        help="write only this fixture (the others are left as they are)")
    args = parser.parse_args()
    if not args.reference:
        parser.error("give the reference checkout with --reference or BAG_REFERENCE_ROOT")
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, os.path.join(args.reference, "src"))
    import torch
    import bag_triton
    from bag_triton import bag as bagmod

    class DeviceTagged(torch.Tensor):
        """CPU tensor that passes the reference's CUDA-device checks."""

        @property
        def is_cuda(self):  # noqa: D401
            return True

    def tag(t):
        return t.as_subclass(DeviceTagged) if isinstance(t, torch.Tensor) else t

    def workspace(a, b, out, grouped):
        ws = bagmod.allocate_bag_workspace(a, b, out, multistream=False, grouped=grouped)
        return bagmod.BagWorkspace(*[tag(x) for x in ws])

    def to_dev(x, layout):
        t = torch.from_numpy(np.ascontiguousarray(x))
        if layout == "col":
            t = torch.from_numpy(np.asfortranarray(x))
        return tag(t)

    # BASELINE config 1 on its exact inputs (bench.make_inputs).
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from bench import CONFIGS, make_inputs
    a, b = make_inputs(dict(CONFIGS["cfg1"]))
    ta, tb = to_dev(a, "row"), to_dev(b, "row")
    out = to_dev(np.zeros(a.shape, np.float32), "row")
    ws = workspace(ta, tb, out, grouped=True)   # schedule "auto" is grouped up to N=8192
    t0 = time.time()
    bag_triton.bag_matmul(ta, tb, out=out, workspace=ws)
    dt = time.time() - t0
    got = out.as_subclass(torch.Tensor).contiguous().numpy().copy()
    np.savez_compressed(os.path.join(HERE, "cfg1_triton_bag_n512.npz"), out=got,
                        a_head=a.ravel()[:64].copy(), b_head=b.ravel()[:64].copy(), n=512,
                        layout="row", schedule="auto", seed=0, dist="uniform(-1,1)")
    cfg1_line = (f"cfg1_triton_bag_n512: BASELINE cfg1 inputs (default_rng(0), U[-1,1), "
                 f"A then B), n=512 layout=row schedule=auto (grouped) {dt:.2f}s")
    print(cfg1_line, flush=True)
    if args.only == "cfg1":
        path = os.path.join(HERE, "MANIFEST.txt")
        lines = [ln for ln in open(path).read().splitlines()
                 if not ln.startswith("cfg1_triton_bag_n512:")]
        with open(path, "w") as f:
            f.write("\n".join(lines + [cfg1_line]) + "\n")
        return

    manifest = [cfg1_line]
    for name, n, layout, schedule, seed, dist in BAG_CASES:
        rng = np.random.default_rng(seed)
        a = _inputs(rng, (n, n), dist)
        b = _inputs(rng, (n, n), dist)
        ta, tb = to_dev(a, layout), to_dev(b, layout)
        out = to_dev(np.zeros((n, n), np.float32), layout)
        ws = workspace(ta, tb, out, grouped=schedule == "grouped")
        t0 = time.time()
        bag_triton.bag_matmul(ta, tb, out=out, workspace=ws, schedule=schedule)
        dt = time.time() - t0
        got = out.as_subclass(torch.Tensor).contiguous().numpy().copy()
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), a=a, b=b, out=got,
                            n=n, layout=layout, schedule=schedule, seed=seed, dist=dist)
        manifest.append(f"{name}: n={n} layout={layout} schedule={schedule} seed={seed} {dt:.2f}s")
        print(manifest[-1], flush=True)

    for idx, (shape, coeffs) in enumerate(PRIMITIVE_CASES):
        m, n, k = shape
        delta, eps, gd, ge = coeffs
        rng = np.random.default_rng(2000 + idx)
        x = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        y = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        v = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        w = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        d = rng.uniform(-1, 1, (m, n)).astype(np.float32)
        e = rng.uniform(-1, 1, (m, n)).astype(np.float32)
        tx, tv = to_dev(x, "row"), to_dev(v, "row")
        ty = to_dev(y, "row") if delta else None
        tw = to_dev(w, "row") if eps else None
        td = to_dev(d.copy(), "row") if gd else None
        te = to_dev(e.copy(), "row") if ge else None
        bag_triton.bag_primitive(tx, ty, tv, tw, td, te, delta=delta, epsilon=eps,
                                 gamma_d=gd, gamma_e=ge)
        d_out = td.as_subclass(torch.Tensor).numpy().copy() if td is not None else d
        e_out = te.as_subclass(torch.Tensor).numpy().copy() if te is not None else e
        name = f"prim_{m}x{n}x{k}_{'_'.join(str(c) for c in coeffs)}".replace("-", "m")
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), x=x, y=y, v=v, w=w, d=d, e=e,
                            d_out=d_out, e_out=e_out, coeffs=np.array(coeffs))
        manifest.append(f"{name}: shape={shape} coeffs={coeffs}")
        print(manifest[-1], flush=True)

    with open(os.path.join(HERE, "MANIFEST.txt"), "w") as f:
        f.write("Generated by tests/golden/make_golden.py from the reference's Triton code\n"
                "(src/bag_triton, TRITON_INTERPRET=1, CPU).\n")
        f.write("\n".join(manifest) + "\n")


if __name__ == "__main__":
    main()
