"""CPU oracle for the BAG (alternative-basis Strassen-Winograd) FP32 matmul.

TEST INFRASTRUCTURE ONLY.  This module is a checker: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs may import it.
The product path (``bag_b200`` and ``libbag_b200.so``) never calls it and has
no CPU fallback.

It restates the reference algorithm (liuyao0322/bag) in numpy, following the
reference's own evaluation order so that transformed operands round exactly as
the reference's do:

* ``bag_matmul``       -- ``include/bag/cuda/bag.cuh:57-245`` (prepare, the seven
                          products, ``prepare_child``/``merge_child`` recursion,
                          decode) for the Minimal and Full bases at any depth.
* ``strassen_one_level`` -- ``include/bag/cuda/strassen.cuh:131-153`` (classic
                          Strassen-1969 comparator, all additions fused).
* ``primitive``        -- ``src/bag_triton/primitive.py:256-461`` and
                          ``include/bag/cuda/strassen.cuh:68-70`` semantics
                          (``(x+delta*y)(v+eps*w)``, gamma codes +-1 / +-2).
* ``hash_value``       -- the reference benchmarks' deterministic input
                          generator, ``benchmarks/cuda/fp32_baseline.cu:26-32``.
* ``validate``         -- the FP64 sampled validator of
                          ``benchmarks/cuda/fp32_baseline.cu:121-192``.

Leaf products use numpy's FP32 GEMM, whose summation order differs from the
reference's sequential ``fmaf`` chain; the bit-exact sequential chain lives in
``oracle/exact_gemm.c`` (``exact_primitive`` below).

Parity pin: ``tests/golden/`` holds outputs of the reference's own Triton
``bag_matmul``/``bag_primitive`` run under ``TRITON_INTERPRET=1`` on seeded
inputs (script: ``tests/golden/make_golden.py``); ``tests/test_oracle.py``
checks this module against them.  On the GPU box the reference's CUDA BAG,
compiled from its headers into ``oracle/_ref/``, pins it again.

Matrices here are logical 2-D arrays; quadrant names follow the reference's
column-major pointer offsets (``bag.cuh:59-65``): ``p`` = X11, ``p+s`` = X21,
``p+col`` = X12, ``p+diag`` = X22.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

F32 = np.float32

# Quadrant indices used by every table below.
Q11, Q12, Q21, Q22 = 0, 1, 2, 3


def quadrants(x: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """Return views (X11, X12, X21, X22) of an even-sized matrix."""
    r, c = x.shape
    if r % 2 or c % 2:
        raise ValueError(f"quadrant split needs even extents, got {x.shape}")
    h, w = r // 2, c // 2
    return x[:h, :w], x[:h, w:], x[h:, :w], x[h:, w:]


def _add(x: np.ndarray, y: np.ndarray, coeff: int) -> np.ndarray:
    """``x + coeff*y`` rounded once in FP32 (coeff in {-1, 0, 1})."""
    if coeff == 0:
        return x.astype(F32, copy=True)
    if coeff == 1:
        return (x.astype(F32) + y.astype(F32)).astype(F32)
    if coeff == -1:
        return (x.astype(F32) - y.astype(F32)).astype(F32)
    raise ValueError(f"coefficient must be -1, 0 or 1, got {coeff}")


def _mm32(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    return np.matmul(x.astype(F32), y.astype(F32)).astype(F32)


# ---------------------------------------------------------------------------
# The BAG coefficient tables (one recursion level).
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class Operand:
    """One product's pointers and primitive coefficients at one level.

    ``x``/``y``/``v``/``w`` name either an input quadrant (``"a11"`` ...) or a
    transformed block (``"sa"``, ``"sb"``, ``"ta12"`` ...); ``d``/``e`` name
    T-basis output quadrants.  Mirrors ``bag_cuda::operands`` and the
    ``submit<D,E,GD,GE>`` codes in ``product`` (``bag.cuh:95-122,165-192``).
    """

    x: str
    y: str
    v: str
    w: str
    d: int
    e: int
    delta: int
    eps: int
    gd: int
    ge: int


# Minimal basis, bag.cuh:112-120 (pointers) and bag.cuh:170-190 (codes).
MINIMAL_OPERANDS: tuple[Operand, ...] = (
    Operand("a12", "a22", "b12", "b22", Q22, Q22, 1, 1, 1, 0),
    Operand("a22", "a21", "b22", "b21", Q21, Q21, -1, -1, 1, 0),
    Operand("sa", "sa", "sb", "sb", Q12, Q12, 0, 0, 1, 0),
    Operand("a11", "a11", "b11", "b11", Q11, Q11, 0, 0, 1, 0),
    Operand("a12", "a12", "b21", "b21", Q11, Q12, 0, 0, 1, 1),
    Operand("sa", "a11", "b12", "b12", Q12, Q22, -1, 0, -1, -1),
    Operand("a21", "a21", "sb", "b11", Q12, Q21, 0, -1, 1, 1),
)

# Full basis, bag.cuh:101-110 (pointers) and bag.cuh:170-190 (codes).
FULL_OPERANDS: tuple[Operand, ...] = (
    Operand("ta22", "ta22", "tb22", "tb22", Q22, Q22, 0, 0, 1, 0),
    Operand("ta21", "ta21", "tb21", "tb21", Q21, Q21, 0, 0, 1, 0),
    Operand("ta12", "ta12", "tb12", "tb12", Q12, Q12, 0, 0, 1, 0),
    Operand("ta11", "ta11", "tb11", "tb11", Q11, Q11, 0, 0, 1, 0),
    Operand("ta12", "ta21", "tb22", "tb12", Q11, Q12, -1, -1, 1, 1),
    Operand("ta12", "ta11", "tb12", "tb21", Q12, Q22, -1, -1, -1, -1),
    Operand("ta22", "ta12", "tb12", "tb11", Q12, Q21, -1, -1, 1, 1),
)


def _minimal_prepare(a: np.ndarray, b: np.ndarray) -> dict[str, np.ndarray]:
    """Forward transform, Minimal basis (``bag.cuh:69-73``): SA, SB only."""
    a11, a12, a21, a22 = quadrants(a)
    b11, b12, b21, b22 = quadrants(b)
    sa = ((a12 - a21).astype(F32) + a22).astype(F32)
    sb = ((b12 - b21).astype(F32) + b22).astype(F32)
    return {"a11": a11, "a12": a12, "a21": a21, "a22": a22,
            "b11": b11, "b12": b12, "b21": b21, "b22": b22, "sa": sa, "sb": sb}


def _full_prepare(a: np.ndarray, b: np.ndarray) -> dict[str, np.ndarray]:
    """Forward transform, Full basis (``bag.cuh:66-68``)."""
    out: dict[str, np.ndarray] = {}
    for name, x in (("a", a), ("b", b)):
        x11, x12, x21, x22 = quadrants(x)
        out[f"t{name}11"] = x11.astype(F32, copy=True)
        out[f"t{name}12"] = (((x12 - x21).astype(F32)) + x22).astype(F32)
        out[f"t{name}21"] = (x22 - x21).astype(F32)
        out[f"t{name}22"] = (x12 + x22).astype(F32)
    return out


def _decode(t: list[np.ndarray]) -> tuple[np.ndarray, ...]:
    """Inverse transform (``bag.cuh:85-86``): T=(x,y,z,w) -> C quadrant updates."""
    x, y, z, w = t
    v11 = x
    v12 = (y - z).astype(F32)
    v21 = (-y + w).astype(F32)
    v22 = ((-y + z).astype(F32) + w).astype(F32)
    return v11, v12, v21, v22


def bag_product(a: np.ndarray, b: np.ndarray, depth: int, basis: str = "minimal",
                leaf: str = "blas") -> np.ndarray:
    """Return A@B computed by ``depth`` BAG levels, reference evaluation order.

    ``leaf="blas"`` computes leaf products with numpy's FP32 GEMM (fast);
    ``leaf="fmaf"`` uses the sequential fmaf chain of ``oracle/exact_gemm.c``,
    the summation order of the reference's CUDA kernels, so the result carries
    the reference CUDA BAG's rounding error (small sizes only).

    This is ``bag_cuda::run<false>`` (``bag.cuh:241-245``): T is zeroed by
    prepare, products accumulate into T in product order 0..6, and decode
    overwrites the result.  Deeper levels materialise the child operands
    ``x+delta*y`` / ``v+eps*w`` exactly as ``prepare_child`` does
    (``bag.cuh:124-135``) and merge ``GD*m`` / ``GE*m`` into T
    (``merge_child``, ``bag.cuh:136-145``).
    """
    if depth < 1:
        raise ValueError("BAG depth must be positive")
    m, k = a.shape
    if b.shape[0] != k:
        raise ValueError(f"inner extents differ: {a.shape} @ {b.shape}")
    n = b.shape[1]
    if m % 2 or k % 2 or n % 2:
        raise ValueError("each BAG level needs even extents")
    full = basis == "full"
    if basis not in ("minimal", "full"):
        raise ValueError(f"basis must be 'minimal' or 'full', got {basis!r}")
    blocks = _full_prepare(a, b) if full else _minimal_prepare(a, b)
    t = [np.zeros((m // 2, n // 2), F32) for _ in range(4)]
    table = FULL_OPERANDS if full else MINIMAL_OPERANDS
    for op in table:
        left = _add(blocks[op.x], blocks[op.y], op.delta)
        right = _add(blocks[op.v], blocks[op.w], op.eps)
        if depth == 1:
            prod = (exact_primitive(left, None, right, None, 0, 0) if leaf == "fmaf"
                    else _mm32(left, right))
        else:
            prod = bag_product(left, right, depth - 1, basis, leaf)
        if op.gd:
            t[op.d] = (t[op.d] + F32(op.gd) * prod).astype(F32)
        if op.ge:
            t[op.e] = (t[op.e] + F32(op.ge) * prod).astype(F32)
    v11, v12, v21, v22 = _decode(t)
    h, w = m // 2, n // 2
    out = np.empty((m, n), F32)
    out[:h, :w], out[:h, w:], out[h:, :w], out[h:, w:] = v11, v12, v21, v22
    return out


def bag_matmul(a: np.ndarray, b: np.ndarray, c: np.ndarray | None = None, *,
               depth: int = 1, basis: str = "minimal") -> np.ndarray:
    """``C + A@B`` by BAG (``bag_cuda::matmul`` semantics, ``bag.cuh:247-260``).

    The top level accumulates the decoded result into C (``decode<true>``,
    ``bag.cuh:88``).  Returns a new array; ``c=None`` means C starts at zero.
    """
    n = a.shape[0]
    size = n
    for _ in range(depth):
        if size <= 0 or size % 2:
            raise ValueError("each BAG level requires an even size")
        size //= 2
    prod = bag_product(a.astype(F32), b.astype(F32), depth, basis)
    if c is None:
        return prod
    return (c.astype(F32) + prod).astype(F32)


# Classic Strassen-1969 one level: strassen.cuh:131-141 (pointers) and
# strassen.cuh:143-153 (codes).  Entries: x, y, v, w, d, e, delta, eps, gd, ge.
STRASSEN_OPERANDS: tuple[tuple, ...] = (
    ("a21", "a22", "b11", "b11", Q21, Q22, 1, 0, 1, -1),
    ("a11", "a12", "b22", "b22", Q12, Q11, 1, 0, 1, -1),
    ("a21", "a11", "b11", "b12", Q22, Q22, -1, 1, 0, 1),
    ("a12", "a22", "b21", "b22", Q11, Q11, -1, 1, 1, 0),
    ("a11", "a11", "b12", "b22", Q12, Q22, 0, -1, 1, 1),
    ("a22", "a22", "b21", "b11", Q11, Q21, 0, -1, 1, 1),
    ("a11", "a22", "b11", "b22", Q11, Q22, 1, 1, 1, 1),
)


def strassen_one_level(a: np.ndarray, b: np.ndarray, c: np.ndarray | None = None) -> np.ndarray:
    """``C + A@B`` by one level of classic Strassen (``strassen_cuda::one_level``).

    Every product accumulates straight into C through the primitive epilogue
    (``strassen.cuh:223-224``); the oracle applies them in product order.
    """
    n = a.shape[0]
    if n % 2:
        raise ValueError("one_level needs an even size")
    a11, a12, a21, a22 = quadrants(a.astype(F32))
    b11, b12, b21, b22 = quadrants(b.astype(F32))
    blocks = {"a11": a11, "a12": a12, "a21": a21, "a22": a22,
              "b11": b11, "b12": b12, "b21": b21, "b22": b22}
    out = np.zeros((n, n), F32) if c is None else c.astype(F32, copy=True)
    cq = list(quadrants(out))
    for x, y, v, w, d, e, delta, eps, gd, ge in STRASSEN_OPERANDS:
        m = _mm32(_add(blocks[x], blocks[y], delta), _add(blocks[v], blocks[w], eps))
        if gd:
            cq[d][...] = (cq[d] + F32(gd) * m).astype(F32)
        if ge:
            cq[e][...] = (cq[e] + F32(ge) * m).astype(F32)
    return out


def winograd_product(a: np.ndarray, b: np.ndarray, depth: int) -> np.ndarray:
    """``A@B`` by ``depth`` levels of Strassen-Winograd, the published
    15-addition form (S. Winograd 1971; e.g. Boyer et al. 2009, Table 1):

    S1 = A21+A22, S2 = S1-A11, S3 = A11-A21, S4 = A12-S2,
    T1 = B12-B11, T2 = B22-T1, T3 = B22-B12, T4 = T2-B21,
    M1 = A11 B11, M2 = A12 B21, M3 = S4 B22, M4 = A22 T4, M5 = S1 T1,
    M6 = S2 T2, M7 = S3 T3, U2 = M1+M6, U3 = U2+M7, U4 = U2+M5,
    C11 = M1+M2, C12 = U4+M3, C21 = U3-M4, C22 = U3+M5,

    each intermediate rounded to FP32, leaves by numpy FP32 GEMM.  The
    reference has no Winograd variant; this is the checker for this build's
    ``BAG_BASIS_WINOGRAD``.
    """
    a = a.astype(F32)
    b = b.astype(F32)
    if depth == 0:
        return _mm32(a, b)
    m, k = a.shape
    n = b.shape[1]
    if m % 2 or k % 2 or n % 2:
        raise ValueError("each level needs even extents")
    a11, a12, a21, a22 = quadrants(a)
    b11, b12, b21, b22 = quadrants(b)
    s1 = (a21 + a22).astype(F32)
    s2 = (s1 - a11).astype(F32)
    s3 = (a11 - a21).astype(F32)
    s4 = (a12 - s2).astype(F32)
    t1 = (b12 - b11).astype(F32)
    t2 = (b22 - t1).astype(F32)
    t3 = (b22 - b12).astype(F32)
    t4 = (t2 - b21).astype(F32)
    mm = lambda x, y: winograd_product(x, y, depth - 1)  # noqa: E731
    m1, m2, m3, m4 = mm(a11, b11), mm(a12, b21), mm(s4, b22), mm(a22, t4)
    m5, m6, m7 = mm(s1, t1), mm(s2, t2), mm(s3, t3)
    u2 = (m1 + m6).astype(F32)
    u3 = (u2 + m7).astype(F32)
    u4 = (u2 + m5).astype(F32)
    out = np.empty((m, n), F32)
    h, w = m // 2, n // 2
    out[:h, :w] = m1 + m2
    out[:h, w:] = u4 + m3
    out[h:, :w] = u3 - m4
    out[h:, w:] = u3 + m5
    return out


def primitive(x, y, v, w, d, e, *, delta: int, eps: int, gamma_d: int, gamma_e: int):
    """The BAG primitive on numpy arrays, returning new (d, e).

    ``product = (x + delta*y) @ (v + eps*w)``; gamma +-1 accumulates,
    +-2 overwrites, 0 leaves the output untouched
    (``src/bag_triton/primitive.py:1-18``).
    """
    left = x if delta == 0 else _add(x, y, delta)
    right = v if eps == 0 else _add(v, w, eps)
    prod = _mm32(left, right)

    def apply(out, gamma):
        if out is None or gamma == 0:
            return None if out is None else out.copy()
        if gamma in (1, -1):
            return (out.astype(F32) + F32(gamma) * prod).astype(F32)
        if gamma in (2, -2):
            return (F32(gamma // 2) * prod).astype(F32)
        raise ValueError(f"gamma must be in -2..2, got {gamma}")

    return apply(d, gamma_d), apply(e, gamma_e)


# ---------------------------------------------------------------------------
# Error metrics and the reference benchmarks' validator.
# ---------------------------------------------------------------------------

def fp64_matmul(a: np.ndarray, b: np.ndarray, c: np.ndarray | None = None) -> np.ndarray:
    """Classical FP64 GEMM, the error oracle named by the benchmark configs."""
    prod = a.astype(np.float64) @ b.astype(np.float64)
    return prod if c is None else c.astype(np.float64) + prod


def rel_frobenius(got: np.ndarray, ref: np.ndarray) -> float:
    """``||got - ref||_F / ||ref||_F`` evaluated in FP64."""
    ref = np.asarray(ref, np.float64)
    diff = np.asarray(got, np.float64) - ref
    return float(np.linalg.norm(diff) / max(np.linalg.norm(ref), 1e-300))


def _mix(x: np.ndarray) -> np.ndarray:
    """32-bit integer hash of ``fp32_baseline.cu:26-29``."""
    x = x.astype(np.uint32)
    x ^= x >> np.uint32(16)
    x = (x * np.uint32(0x7FEB352D)).astype(np.uint32)
    x ^= x >> np.uint32(15)
    x = (x * np.uint32(0x846CA68B)).astype(np.uint32)
    return x ^ (x >> np.uint32(16))


def hash_value(index: np.ndarray, seed: int) -> np.ndarray:
    """Exactly representable inputs in [-0.5, 0.5), ``fp32_baseline.cu:30-32``."""
    idx = np.asarray(index, dtype=np.uint64).astype(np.uint32)  # uint32_t(i) truncation
    h = _mix(idx ^ np.uint32(seed & 0xFFFFFFFF))
    return ((h & np.uint32(65535)).astype(np.int64) - 32768).astype(F32) * F32(1.0 / 65536.0)


def hash_matrix(rows: int, cols: int, seed: int, ld: int | None = None) -> np.ndarray:
    """Column-major N x N matrix filled like the reference's ``initialize``.

    Element (r, c) holds ``value(r + c*ld, seed)`` (``fp32_baseline.cu:33-36``).
    """
    ld = rows if ld is None else ld
    r = np.arange(rows, dtype=np.uint64)[:, None]
    c = np.arange(cols, dtype=np.uint64)[None, :]
    return hash_value(r + c * np.uint64(ld), seed)


@dataclass
class ValidationResult:
    relative_l2: float
    max_abs: float
    max_scaled: float
    count: int
    passed: bool


def validate(c_got: np.ndarray, a: np.ndarray, b: np.ndarray, c0: np.ndarray, repeats: int,
             samples: int = 128, seed: int = 0) -> ValidationResult:
    """FP64 sampled validation of ``C = C0 + repeats*A@B``.

    Restates ``fp32_baseline.cu:121-192`` for a whole-matrix case: exhaustive
    for N <= 128, otherwise the four corners plus ``samples`` random positions;
    pass iff every checked value is finite, ``relative_l2 <= 3e-5`` and
    ``max_abs/(1+max|ref|) <= 1e-4``.
    """
    n_rows, n_cols = c_got.shape
    if n_rows <= 128 and n_cols <= 128:
        rows, cols = np.meshgrid(np.arange(n_rows), np.arange(n_cols), indexing="ij")
        rows, cols = rows.ravel(), cols.ravel()
    else:
        rng = np.random.RandomState(20261017 + n_rows + seed)
        pos = {(0, 0), (n_rows - 1, 0), (0, n_cols - 1), (n_rows - 1, n_cols - 1)}
        while len(pos) < samples:
            pos.add((int(rng.randint(n_rows)), int(rng.randint(n_cols))))
        rows = np.array([p[0] for p in sorted(pos)])
        cols = np.array([p[1] for p in sorted(pos)])
    a64 = a.astype(np.float64)
    b64 = b.astype(np.float64)
    dots = np.einsum("ik,ki->i", a64[rows, :], b64[:, cols])
    ref = c0.astype(np.float64)[rows, cols] + repeats * dots
    got = c_got[rows, cols].astype(np.float64)
    d = np.abs(got - ref)
    finite = bool(np.all(np.isfinite(got)))
    rel = float(np.sqrt(np.sum(d * d) / max(np.sum(ref * ref), 1e-300)))
    max_abs = float(d.max()) if d.size else 0.0
    max_scaled = max_abs / (1.0 + float(np.abs(ref).max()))
    ok = finite and rel <= 3e-5 and max_scaled <= 1e-4
    return ValidationResult(rel, max_abs, max_scaled, int(got.size), ok)


# ---------------------------------------------------------------------------
# Seeded benchmark inputs (the configs in BASELINE.json; row-major A then B).
# ---------------------------------------------------------------------------

def config_inputs(m: int, k: int, n: int, seed: int, dist: str) -> tuple[np.ndarray, np.ndarray]:
    """A (m x k) then B (k x n), row-major FP32, ``numpy.random.default_rng(seed)``."""
    rng = np.random.default_rng(seed)
    if dist == "uniform_pm1":
        a = rng.uniform(-1.0, 1.0, (m, k)).astype(F32)
        b = rng.uniform(-1.0, 1.0, (k, n)).astype(F32)
    elif dist == "uniform_01":
        a = rng.uniform(0.0, 1.0, (m, k)).astype(F32)
        b = rng.uniform(0.0, 1.0, (k, n)).astype(F32)
    elif dist == "normal":
        a = rng.standard_normal((m, k), dtype=F32)
        b = rng.standard_normal((k, n), dtype=F32)
    else:
        raise ValueError(f"unknown distribution {dist!r}")
    return a, b


# ---------------------------------------------------------------------------
# The exact (sequential fmaf) primitive, from oracle/exact_gemm.c.
# ---------------------------------------------------------------------------

_HERE = os.path.dirname(os.path.abspath(__file__))
_EXACT_SO = os.path.join(_HERE, "_build", "liboracle_exact.so")
_exact_lib = None


def build_exact(force: bool = False) -> str:
    """Compile ``oracle/exact_gemm.c`` with gcc (no FP contraction)."""
    import subprocess
    src = os.path.join(_HERE, "exact_gemm.c")
    os.makedirs(os.path.dirname(_EXACT_SO), exist_ok=True)
    if force or not os.path.exists(_EXACT_SO) or os.path.getmtime(_EXACT_SO) < os.path.getmtime(src):
        subprocess.check_call(["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC",
                               "-shared", "-o", _EXACT_SO, src, "-lm"])
    return _EXACT_SO


def _lib():
    global _exact_lib
    if _exact_lib is None:
        _exact_lib = ctypes.CDLL(build_exact())
        fn = _exact_lib.oracle_primitive_exact
        fn.restype = None
        fn.argtypes = [ctypes.c_int] * 3 + [ctypes.c_void_p] * 4 + [ctypes.c_int] * 6 + \
            [ctypes.c_void_p, ctypes.c_int]
    return _exact_lib


def exact_primitive(x: np.ndarray, y: np.ndarray | None, v: np.ndarray, w: np.ndarray | None,
                    delta: int, eps: int) -> np.ndarray:
    """``(x+delta*y)@(v+eps*w)`` with every output a sequential ``fmaf`` chain.

    k runs in ascending order from a zero accumulator, the order of the
    reference's SIMT kernels (``simt.cuh:136-159``), so single-writer outputs
    of a correct CUDA primitive match this bit for bit.
    """
    m, k = x.shape
    n = v.shape[1]
    cm = lambda t: np.asfortranarray(t, dtype=F32)  # noqa: E731
    xf, vf = cm(x), cm(v)
    yf = cm(y) if y is not None else xf
    wf = cm(w) if w is not None else vf
    out = np.zeros((m, n), F32, order="F")
    ptr = lambda t: t.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    _lib().oracle_primitive_exact(m, n, k, ptr(xf), ptr(yf), ptr(vf), ptr(wf),
                                  max(m, 1), max(m, 1), max(k, 1), max(k, 1), delta, eps,
                                  ptr(out), max(m, 1))
    return np.ascontiguousarray(out)
