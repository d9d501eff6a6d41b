"""The CPU oracle (oracle/bn254_oracle.c) pinned against golden vectors made
by the reference's own arithmetic (tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest

import pyoracle as O
from conftest import GOLDEN


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def test_mt19937_64_known_answer():
    # 10000th output of std::mt19937_64 with the default seed 5489 (C++11 [rand.predef])
    r = O.Rng(5489)
    for _ in range(9999):
        r.next()
    assert r.next() == 9981545732273789042


def test_field_ops_match_reference():
    g = load("field.npz")
    a, b = g["a"], g["b"]
    for i in range(a.shape[0]):
        assert np.array_equal(O.fr_mul(a[i], b[i]), g["fr_mul"][i])
        assert np.array_equal(O.fp_mul(a[i], b[i]), g["fp_mul"][i])
    assert O.fr_to_int(g["fr_one"]) == 1
    assert O.fp_to_int(g["fp_one"]) == 1


def test_omega_matches_reference_for_all_sizes():
    g = load("omega.npz")
    for ln in range(29):
        assert np.array_equal(O.compute_omega(ln, False), g["fwd"][ln])
        assert np.array_equal(O.compute_omega(ln, True), g["inv"][ln])
    # w is a primitive 2^28-th root: w^(2^27) = -1
    w = g["fwd"][28]
    x = w.copy()
    for _ in range(27):
        x = O.fr_mul(x, x)
    assert O.fr_to_int(x) == O.R - 1


def _cases(g, suffix="_result"):
    return sorted(k[: -len(suffix)] for k in g.files if k.endswith(suffix))


def test_g1_msm_oracle_matches_reference():
    g = load("g1_msm.npz")
    for name in _cases(g):
        pts, sc, res = g[name + "_points"], g[name + "_scalars"], g[name + "_result"]
        assert np.array_equal(O.msm_g1(pts, sc), res), name
        assert np.array_equal(O.msm_g1(pts, sc, nthreads=4), res), name
        assert np.array_equal(O.msm_g1_naive(pts, sc), res), name


def test_g2_msm_oracle_matches_reference():
    g = load("g2_msm.npz")
    for name in _cases(g):
        pts, sc, res = g[name + "_points"], g[name + "_scalars"], g[name + "_result"]
        assert np.array_equal(O.msm_g2(pts, sc), res), name
        assert np.array_equal(O.msm_g2_naive(pts, sc), res), name
        if res.any():
            assert O.g2_on_curve(res)


def test_ntt_oracle_matches_reference():
    g = load("ntt.npz")
    for name in _cases(g, "_fwd"):
        x, ln = g[name + "_in"], int(g[name + "_log"][0])
        assert np.array_equal(O.ntt(x, ln, False), g[name + "_fwd"]), name
        assert np.array_equal(O.ntt(x, ln, True), g[name + "_inv"]), name
        assert np.array_equal(O.ntt(O.ntt(x, ln, False), ln, True), x), name


def test_pippenger_equals_naive_larger():
    rng = O.Rng(77)
    k = rng.fr_vector(3000)
    pts = O.g1_fixed_base(k)
    sc = rng.fr_vector(3000)
    assert np.array_equal(O.msm_g1(pts, sc, nthreads=8), O.msm_g1_naive(pts, sc))


def _poly_eval(coeffs, x):
    acc = 0
    for c in reversed([O.fr_to_int(v) for v in coeffs]):
        acc = (acc * x + c) % O.R
    return acc


@pytest.mark.parametrize("ln", [2, 5, 9])
def test_compute_h_divides(ln):
    """A(x)B(x) - C(x) = h(x)(x^n - 1) at a random point when C = A*B on the domain."""
    n = 1 << ln
    rng = O.Rng(1000 + ln)
    a, b = rng.fr_vector(n), rng.fr_vector(n)
    c = np.stack([O.fr_mul(a[i], b[i]) for i in range(n)])
    h = O.compute_h_from_evals(a, b, c, ln)
    A, B, C = (O.ntt(v, ln, True) for v in (a, b, c))
    tau = 0x1234567890ABCDEF1234567 % O.R
    lhs = (_poly_eval(A, tau) * _poly_eval(B, tau) - _poly_eval(C, tau)) % O.R
    rhs = _poly_eval(h, tau) * (pow(tau, n, O.R) - 1) % O.R
    assert lhs == rhs
    assert O.fr_to_int(h[n - 1]) == 0  # deg h <= n - 2


def test_fixed_base_matches_reference_scalar_mul():
    if not O.ref_available():
        pytest.skip("reference arithmetic library not built here")
    import ctypes
    ref = O.ref()
    rng = O.Rng(5)
    k = rng.fr_vector(8)
    pts = O.g1_fixed_base(k)
    g = O.g1_generator()
    inf = ctypes.c_int()
    for i in range(8):
        o = np.zeros(8, np.uint64)
        ref.ref_g1_scalar_mul(o.ctypes.data_as(O._u64p), ctypes.byref(inf), g.ctypes.data_as(O._u64p), 0,
                              np.ascontiguousarray(k[i]).ctypes.data_as(O._u64p))
        assert np.array_equal(o, pts[i])
