"""GPU parity of the NTT / INTT / coset NTT and compute_h against the
reference-pinned oracle, bit-exact."""
import os

import numpy as np
import pytest

import pyoracle as O
import zkml_b200 as Z
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a):
    return Z.to_device(a)


def test_golden_vectors():
    gz = np.load(os.path.join(GOLDEN, "ntt.npz"))
    names = sorted(k[:-4] for k in gz.files if k.endswith("_fwd"))
    for name in names:
        x, ln = gz[name + "_in"], int(gz[name + "_log"][0])
        for inv, key in ((False, "_fwd"), (True, "_inv")):
            assert np.array_equal(Z.to_host(Z.ntt(dev(x), ln, inv)), gz[name + key]), (name, inv)
            # reference-shaped entry point (synchronous, out-of-place and in place)
            d_in, d_out = dev(x), torch.empty_like(dev(x))
            assert Z.ntt_ref(d_out, d_in, ln, inv) == Z.ZK_OK
            assert np.array_equal(Z.to_host(d_out), gz[name + key]), (name, inv)
            assert Z.ntt_ref(d_in, d_in, ln, inv) == Z.ZK_OK
            assert np.array_equal(Z.to_host(d_in), gz[name + key]), (name, inv)


@pytest.mark.parametrize("ln", [6, 9, 11, 12, 13, 16, 17])
def test_matches_oracle(ln):
    x = O.Rng(ln).fr_vector(1 << ln)
    d = dev(x)
    assert np.array_equal(Z.to_host(Z.ntt(d, ln, False)), O.ntt(x, ln, False))
    assert np.array_equal(Z.to_host(Z.ntt(d, ln, True)), O.ntt(x, ln, True))


@pytest.mark.parametrize("ln", [4, 10, 13, 16])
def test_coset_matches_oracle(ln):
    x = O.Rng(50 + ln).fr_vector(1 << ln)
    for gval in (Z.fr_from_int(5), O.Rng(ln).fr_vector(1)[0]):
        d = dev(x)
        assert np.array_equal(Z.to_host(Z.ntt(d, ln, False, coset=gval)), O.coset_ntt(x, ln, False, gval))
        assert np.array_equal(Z.to_host(Z.ntt(d, ln, True, coset=gval)), O.coset_ntt(x, ln, True, gval))


@pytest.mark.parametrize("ln", [20, 22, 24])
def test_full_size_bit_exact(ln):
    """Config 3's sizes: forward, inverse, coset forward and coset inverse
    (g = 5) over whole vectors, bit-exact against the oracle's restatement of
    the reference's radix-2 transform (its stages split over the host cores),
    plus the round trip INTT(NTT(x)) = x on the device."""
    n = 1 << ln
    cores = os.cpu_count() or 1
    x = Z.random_fr(n, 0xA000 + ln)
    d = dev(x)
    y = Z.ntt(d, ln, False)
    assert np.array_equal(Z.to_host(y), O.ntt(x, ln, False, nthreads=cores)), "forward"
    assert torch.equal(Z.ntt(y, ln, True), d), "round trip"
    assert np.array_equal(Z.to_host(Z.ntt(d, ln, True)), O.ntt(x, ln, True, nthreads=cores)), "inverse"
    g = Z.fr_from_int(5)
    assert np.array_equal(Z.to_host(Z.ntt(d, ln, False, coset=g)), O.coset_ntt(x, ln, False, g, nthreads=cores)), "coset forward"
    assert np.array_equal(Z.to_host(Z.ntt(d, ln, True, coset=g)), O.coset_ntt(x, ln, True, g, nthreads=cores)), "coset inverse"


def test_in_place_and_ranges():
    x = O.Rng(2).fr_vector(1 << 10)
    d = dev(x)
    Z.ntt(d, 10, False, out=d)
    assert np.array_equal(Z.to_host(d), O.ntt(x, 10, False))
    before = d.clone()
    assert Z.ntt_ref(d, d, 25, False) == Z.ZK_ERR_RANGE       # reference limit 2^24: output untouched
    assert torch.equal(before, d)


@pytest.mark.parametrize("ln", [2, 10, 13])
def test_compute_h_matches_oracle(ln):
    n = 1 << ln
    rng = O.Rng(900 + ln)
    a, b, c = rng.fr_vector(n), rng.fr_vector(n), rng.fr_vector(n)
    exp = O.compute_h_from_evals(a, b, c, ln)
    got = Z.compute_h(dev(a), dev(b), dev(c), ln)
    assert np.array_equal(Z.to_host(got), exp)


def test_compute_h_satisfied_divides_at_2_16():
    ln, n = 16, 1 << 16
    a = Z.random_fr(n, 1)
    b = Z.random_fr(n, 2)
    # c = a * b pointwise (a satisfied R1CS): h(x)(x^n - 1) = A(x)B(x) - C(x)
    c = np.stack([O.fr_mul(a[i], b[i]) for i in range(n)])
    h = Z.to_host(Z.compute_h(dev(a), dev(b), dev(c), ln))
    A, B, C = (Z.to_host(Z.ntt(dev(v), ln, True)) for v in (a, b, c))
    tau = O.Rng(3).fr_vector(1)[0]
    lhs = O.fr_mul(O.fr_poly_eval(A, tau), O.fr_poly_eval(B, tau))
    lhs_i = (O.fr_to_int(lhs) - O.fr_to_int(O.fr_poly_eval(C, tau))) % O.R
    rhs_i = O.fr_to_int(O.fr_poly_eval(h, tau)) * (pow(O.fr_to_int(tau), n, O.R) - 1) % O.R
    assert lhs_i == rhs_i
    assert not h[n - 1].any()


@pytest.mark.parametrize("s_log", [0, 1, 2, 3])
def test_ntt_cross_matches_oracle(s_log):
    """The cross-part step of a transform split over 2^s_log parts
    (zk_ntt_cross_device) against the oracle's direct sums, every mode,
    direction and factor, first and last part."""
    from oracle_prover import OracleProver
    L = 10
    n = 1 << L
    m = n >> s_log
    orc = OracleProver({"n": n, "log_n": L, "m": 1, "num_public": 0, "l": 0}, [])
    x = O.Rng(70 + s_log).fr_vector(m)
    g = O.fr_from_int(5)
    for part in sorted({0, (1 << s_log) - 1}):
        for mode in (0, 1):
            for inverse in (False, True):
                for factor, finv in ((None, False), (g, False), (g, True)):
                    got = Z.to_host(Z.ntt_cross(dev(x), L, s_log, part, inverse, mode, factor, finv))
                    exp = orc.cross(torch.from_numpy(x.view(np.int64).copy()), L, s_log, part, inverse, mode, factor,
                                    finv).numpy().view(np.uint64)
                    assert np.array_equal(got, exp), (part, mode, inverse, factor is not None, finv)


def test_ntt_cross_refuses_bad_arguments():
    x = dev(O.Rng(9).fr_vector(256))
    for args in ((8, 4, 0, 0), (8, 5, 0, 0), (8, 2, 4, 0), (8, 2, 0, 2), (8, -1, 0, 0)):
        L, s_log, part, mode = args
        with pytest.raises(Z.ZkError):
            Z.ntt_cross(x, L, s_log, part, False, mode)
    with pytest.raises(Z.ZkError):
        Z.ntt_cross(x, 8, 1, 0, False, 0, out=x)  # in place is refused
