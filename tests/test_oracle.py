"""Pin the CPU oracle against the reference's own outputs (golden fixtures).

The fixtures in ``tests/golden`` come from the reference's Triton
``bag_matmul``/``bag_primitive`` run under ``TRITON_INTERPRET=1``
(``tests/golden/make_golden.py``).  The tolerances are the reference's own:
rel-L2 <= 3e-4 for IEEE BAG (``tests/triton/test_bag.py:60-61``) and
``atol=2e-4+2e-6*k, rtol=2e-4`` for the primitive (``test_primitive.py:89``);
the oracle is also held to a much tighter FP32-level bound.
"""

from __future__ import annotations

import glob
import os

import numpy as np
import pytest

from oracle import bag_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
BAG_FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "bag_*.npz")))
PRIM_FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "prim_*.npz")))


def test_fixtures_present():
    assert len(BAG_FIXTURES) >= 7 and len(PRIM_FIXTURES) >= 7


@pytest.mark.parametrize("path", BAG_FIXTURES, ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_matches_reference_bag(path):
    z = np.load(path)
    a, b, out = z["a"], z["b"], z["out"]
    mine = O.bag_product(a, b, 1, "minimal")
    ref64 = O.fp64_matmul(a, b)
    # Same algorithm, same rounding of every transformed operand; only the
    # Triton kernel's K tiling of the leaf sums differs.
    assert O.rel_frobenius(mine, out) <= 2e-6
    assert O.rel_frobenius(mine, ref64) <= 3e-4            # test_bag.py:60
    n = a.shape[0]
    assert np.abs(mine - ref64).max() <= 2e-3 + 2e-5 * n    # test_bag.py:61


@pytest.mark.parametrize("path", BAG_FIXTURES[:4], ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_bitexact_on_small_serial(path):
    z = np.load(path)
    if str(z["schedule"]) != "serial" or int(z["n"]) > 64:
        pytest.skip("bit-exact only where the Triton leaf runs a single K tile")
    mine = O.bag_product(z["a"], z["b"], 1, "minimal")
    assert np.array_equal(mine, z["out"])


@pytest.mark.parametrize("path", PRIM_FIXTURES, ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_matches_reference_primitive(path):
    z = np.load(path)
    delta, eps, gd, ge = [int(c) for c in z["coeffs"]]
    d, e = O.primitive(z["x"], z["y"], z["v"], z["w"], z["d"], z["e"], delta=delta, eps=eps,
                       gamma_d=gd, gamma_e=ge)
    k = z["x"].shape[1]
    tol = dict(atol=2e-4 + 2e-6 * k, rtol=2e-4)
    np.testing.assert_allclose(d, z["d_out"], **tol)
    np.testing.assert_allclose(e, z["e_out"], **tol)


@pytest.mark.parametrize("path", PRIM_FIXTURES, ids=lambda p: os.path.basename(p)[:-4])
def test_exact_primitive_matches_reference(path):
    z = np.load(path)
    delta, eps, _, _ = [int(c) for c in z["coeffs"]]
    got = O.exact_primitive(z["x"], z["y"] if delta else None, z["v"], z["w"] if eps else None,
                            delta, eps)
    d_ref, _ = O.primitive(z["x"], z["y"], z["v"], z["w"], np.zeros_like(z["d"]), None,
                           delta=delta, eps=eps, gamma_d=2, gamma_e=0)
    k = z["x"].shape[1]
    np.testing.assert_allclose(got, d_ref, atol=2e-4 + 2e-6 * k, rtol=2e-4)


def test_exact_primitive_is_a_sequential_fmaf_chain():
    # Known answer: with exactly representable inputs the chain is exact.
    x = np.array([[1.0, 2.0, 3.0]], np.float32)
    v = np.array([[4.0], [5.0], [6.0]], np.float32)
    assert O.exact_primitive(x, None, v, None, 0, 0)[0, 0] == 32.0
    # A case where one rounding per step is visible: 1 + 2^-24 + 2^-24.
    x = np.array([[1.0, 2.0 ** -24, 2.0 ** -24]], np.float32)
    v = np.ones((3, 1), np.float32)
    assert O.exact_primitive(x, None, v, None, 0, 0)[0, 0] == np.float32(1.0)


@pytest.mark.parametrize("depth", [1, 2, 3])
@pytest.mark.parametrize("basis", ["minimal", "full"])
def test_oracle_depths_against_fp64(depth, basis):
    rng = np.random.default_rng(7 + depth)
    n = 64
    a = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    b = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    c = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    got = O.bag_matmul(a, b, c, depth=depth, basis=basis)
    assert O.rel_frobenius(got, O.fp64_matmul(a, b, c)) < 2e-6 * depth


def test_oracle_strassen_one_level():
    rng = np.random.default_rng(3)
    a, b, c = (rng.uniform(-1, 1, (48, 48)).astype(np.float32) for _ in range(3))
    got = O.strassen_one_level(a, b, c)
    assert O.rel_frobenius(got, O.fp64_matmul(a, b, c)) < 1e-6


def test_hash_generator_known_values():
    # fp32_baseline.cu:26-32: values are multiples of 2^-16 in [-0.5, 0.5).
    v = O.hash_value(np.arange(100000), 11)
    assert v.dtype == np.float32
    assert v.min() >= -0.5 and v.max() < 0.5
    assert np.all(v * 65536 == np.round(v * 65536))
    # mix(0 ^ 11): hand-evaluated from the published hash steps.
    x = 11
    x ^= x >> 16; x = (x * 0x7FEB352D) & 0xFFFFFFFF; x ^= x >> 15
    x = (x * 0x846CA68B) & 0xFFFFFFFF; x ^= x >> 16
    assert v[0] == np.float32(((x & 65535) - 32768) / 65536.0)


def test_validator_semantics():
    n = 96
    a = O.hash_matrix(n, n, 11)
    b = O.hash_matrix(n, n, 23)
    c0 = O.hash_matrix(n, n, 37)
    good = O.bag_matmul(a, b, O.bag_matmul(a, b, c0))   # two accumulating calls
    assert O.validate(good, a, b, c0, repeats=2).passed
    assert not O.validate(good, a, b, c0, repeats=1).passed
    bad = good.copy()
    bad[5, 7] += 1.0
    assert not O.validate(bad, a, b, c0, repeats=2).passed


def test_config_inputs_are_seeded():
    a1, b1 = O.config_inputs(8, 8, 8, 0, "uniform_pm1")
    a2, b2 = O.config_inputs(8, 8, 8, 0, "uniform_pm1")
    assert np.array_equal(a1, a2) and np.array_equal(b1, b2)
    assert a1.dtype == np.float32 and a1.min() >= -1 and a1.max() < 1
    a3, _ = O.config_inputs(8, 8, 8, 2, "normal")
    assert a3.dtype == np.float32


def test_winograd_oracle_is_a_matmul():
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (64, 96)).astype(np.float32)
    b = rng.uniform(-1, 1, (96, 32)).astype(np.float32)
    exact = O.fp64_matmul(a, b)
    for depth in (1, 2, 3):
        assert O.rel_frobenius(O.winograd_product(a, b, depth), exact) < 1e-5


def test_oracle_matches_reference_triton_on_cfg1():
    """BASELINE cfg1 (512, U[-1,1) from default_rng(0), one level): the oracle on the
    exact bench inputs against the reference's Triton bag_matmul on the same inputs."""
    from bench import CONFIGS, make_inputs
    a, b = make_inputs(dict(CONFIGS["cfg1"]))
    z = np.load(os.path.join(GOLDEN, "cfg1_triton_bag_n512.npz"))
    assert np.array_equal(z["a_head"], a.ravel()[:64])
    assert np.array_equal(z["b_head"], b.ravel()[:64])
    ref64 = O.fp64_matmul(a, b)
    assert O.rel_frobenius(z["out"], ref64) <= 3e-4                # test_bag.py:60
    for leaf in ("blas", "fmaf"):
        mine = O.bag_product(a, b, 1, "minimal", leaf=leaf)
        assert O.rel_frobenius(mine, z["out"]) <= 2e-6
        assert O.rel_frobenius(mine, ref64) <= 3e-4
