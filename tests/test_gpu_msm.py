"""GPU parity of the G1/G2 MSM against the reference-pinned oracle.

Bit-exact: every result is the canonical affine point.  Small cases use the
golden vectors made by the reference's own arithmetic; medium sizes compare
with the oracle's Pippenger restatement; full sizes (2^20, 2^24) use the
size-independent identity sum_i s_i (k_i G) = (sum_i s_i k_i) G."""
import os

import numpy as np
import pytest

import pyoracle as O
import zkml_b200 as Z
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def g(name):
    return np.load(os.path.join(GOLDEN, name))


def cases(gz):
    return sorted(k[: -len("_result")] for k in gz.files if k.endswith("_result"))


def dev(a):
    return Z.to_device(a)


def test_device_is_b200():
    assert Z.device_count() >= 1
    assert torch.cuda.get_device_capability(0)[0] >= 10


@pytest.mark.parametrize("path", ["device", "host", "ref"])
def test_g1_golden(path):
    gz = g("g1_msm.npz")
    for name in cases(gz):
        pts, sc, res = gz[name + "_points"], gz[name + "_scalars"], gz[name + "_result"]
        if path == "device":
            out = Z.msm_g1(dev(pts), dev(sc))
        elif path == "host":
            out = Z.msm_g1(pts, sc)
        else:
            jac = Z.msm_g1_ref(Z.packed_to_ref_g1(pts), sc)
            if res.any():
                assert O.fp_to_int(jac[8:12]) == 1, name   # Z = one
                out = jac[:8]
            else:
                assert not jac[:4].any() and not jac[8:].any() and O.fp_to_int(jac[4:8]) == 1, name
                out = np.zeros(8, np.uint64)
        assert np.array_equal(out, res), (path, name)


@pytest.mark.parametrize("path", ["device", "host", "ref"])
def test_g2_golden(path):
    gz = g("g2_msm.npz")
    for name in cases(gz):
        pts, sc, res = gz[name + "_points"], gz[name + "_scalars"], gz[name + "_result"]
        if path == "device":
            out = Z.msm_g2(dev(pts), dev(sc))
        elif path == "host":
            out = Z.msm_g2(pts, sc)
        else:
            jac = Z.msm_g2_ref(Z.packed_to_ref_g2(pts), sc)
            out = jac[:16] if res.any() else np.zeros(16, np.uint64)
        assert np.array_equal(out, res), (path, name)


def test_zero_points_is_identity():
    assert not Z.msm_g1(np.zeros((0, 8), np.uint64), np.zeros((0, 4), np.uint64)).any()
    jac = Z.msm_g1_ref(np.zeros((0, 72), np.uint8), np.zeros((0, 4), np.uint64), n=0)
    assert O.fp_to_int(jac[4:8]) == 1 and not jac[8:].any()


def test_fixed_base_matches_oracle():
    rng = O.Rng(11)
    k = rng.fr_vector(1000)
    k[3] = 0
    got = Z.to_host(Z.g1_fixed_base(dev(k)))
    assert np.array_equal(got, O.g1_fixed_base(k))
    k2 = k[:64]
    got2 = Z.to_host(Z.g2_fixed_base(dev(k2)))
    assert np.array_equal(got2, O.g2_fixed_base(k2))


def _random_instance(n, seed, g2=False):
    rng = O.Rng(seed)
    k = rng.fr_vector(n)
    sc = rng.fr_vector(n)
    kd = dev(k)
    pts = Z.g2_fixed_base(kd) if g2 else Z.g1_fixed_base(kd)
    return k, pts, sc


@pytest.mark.parametrize("n", [255, 256, 257, 1000, 4097, 1 << 14, 1 << 16])
def test_g1_matches_oracle(n):
    _, pts, sc = _random_instance(n, 100 + n)
    exp = O.msm_g1(Z.to_host(pts), sc, nthreads=os.cpu_count())
    assert np.array_equal(Z.msm_g1(pts, dev(sc)), exp)


@pytest.mark.parametrize("c", [3, 7, 11, 13, 16, 18])
def test_g1_window_sizes_agree(c, monkeypatch):
    n = 5000
    _, pts, sc = _random_instance(n, 7)
    exp = O.msm_g1(Z.to_host(pts), sc, nthreads=os.cpu_count())
    monkeypatch.setenv("ZK_MSM_WINDOW_BITS", str(c))
    assert np.array_equal(Z.msm_g1(pts, dev(sc)), exp)


def test_g1_skewed_scalars():
    """Bucket skew: 40% zeros, 30% one repeated scalar, 20% values < 2^16,
    plus duplicated points and P, -P pairs (the benchmark's 10% zero / 10% small
    variant is a milder version of this)."""
    n = 20000
    rng = O.Rng(21)
    k = rng.fr_vector(n)
    sc = rng.fr_vector(n)
    u = np.random.default_rng(5).random(n)
    sc[u < 0.4] = 0
    sc[(u >= 0.4) & (u < 0.7)] = sc[0]
    small = (u >= 0.7) & (u < 0.9)
    for i in np.nonzero(small)[0]:
        sc[i] = O.fr_from_int(int(rng.next() & 0xFFFF))
    pts = Z.to_host(Z.g1_fixed_base(dev(k)))
    pts[100:200] = pts[300:400]          # duplicates
    pts[500:600] = 0                      # infinity
    exp = O.msm_g1(pts, sc, nthreads=os.cpu_count())
    assert np.array_equal(Z.msm_g1(dev(pts), dev(sc)), exp)
    assert np.array_equal(Z.msm_g1(pts, sc), exp)


def test_g1_survey_variant_10pct_zero_10pct_small():
    n = 1 << 16
    k, pts, sc = _random_instance(n, 0x5EED0010)
    perm = np.random.default_rng(0x5EED0010).permutation(n)
    sc[perm[: n // 10]] = 0
    for i in perm[n // 10: n // 5]:
        sc[i] = Z.fr_from_int(int(i) & 0xFFFF)
    exp = O.msm_g1(Z.to_host(pts), sc, nthreads=os.cpu_count())
    assert np.array_equal(Z.msm_g1(pts, dev(sc)), exp)


@pytest.mark.parametrize("log_n", [20, 24])
def test_g1_survey_variant_full_size_identity(log_n):
    """Config 2's skewed variant (10 % zero, 10 % uniform below 2^16, the rest
    uniform, positions shuffled) at 2^20 and 2^24 points: the identity
    sum_i s_i (k_i G) = (sum_i s_i k_i) G, device and host entry points."""
    n = 1 << log_n
    k = Z.random_fr(n, 0x5EED2000 + log_n)
    sc = Z.random_fr(n, 0x5EED3000 + log_n)
    rng = np.random.default_rng(0x5EED0000 + log_n)
    perm = rng.permutation(n)
    sc[perm[: n // 10]] = 0
    small = perm[n // 10: n // 5]
    sc[small] = 0
    sc[small, 0] = rng.integers(0, 1 << 16, small.size).astype(np.uint64)
    sc[small] = O.fr_from_std_vector(sc[small])  # the small values as Montgomery Fr
    pts = Z.g1_fixed_base(dev(k))
    got = Z.msm_g1(pts, dev(sc))
    exp = O.g1_fixed_base(O.fr_dot(k, sc)[None, :])[0]
    assert np.array_equal(got, exp)
    assert np.array_equal(Z.msm_g1(Z.to_host(pts), sc), exp)


@pytest.mark.parametrize("log_n", [20, 24])
def test_g1_full_size_identity(log_n):
    """sum_i s_i (k_i G) == (sum_i s_i k_i) G at the benchmark sizes."""
    n = 1 << log_n
    k = Z.random_fr(n, 0x5EED0000 + log_n)
    sc = Z.random_fr(n, 0x5EED1000 + log_n)
    kd = dev(k)
    pts = Z.g1_fixed_base(kd)
    got = Z.msm_g1(pts, dev(sc))
    dot = O.fr_dot(k, sc)
    exp = O.g1_fixed_base(dot[None, :])[0]
    assert np.array_equal(got, exp)
    # spot-check the generated points themselves
    idx = np.random.default_rng(1).integers(0, n, 64)
    ph = Z.to_host(pts[torch.as_tensor(idx, device=pts.device)])
    assert np.array_equal(ph, O.g1_fixed_base(k[idx]))


@pytest.mark.parametrize("n,skew", [((1 << 20) + 777, False), ((1 << 21) + 3, True)])
def test_g1_host_pipelined_matches_device(n, skew):
    """Host inputs from 2^20 points take the two-batch pipelined path (each
    batch sorted and accumulated while the next one is copied, bucket arrays
    merged): the result equals the device path's and the identity
    sum_i s_i (k_i G) = (sum_i s_i k_i) G."""
    k = Z.random_fr(n, 0x7A00 + n)
    sc = Z.random_fr(n, 0x7B00 + n)
    if skew:  # a witness-like second half: 0/1 scalars and repeats (aggregated atomics, hot buckets)
        rng = np.random.default_rng(n)
        half = n // 2
        tail = np.zeros((n - half, 4), np.uint64)
        tail[rng.random(n - half) < 0.8] = Z.fr_from_int(1)
        tail[:1000] = sc[7]
        sc[half:] = tail
    pts = Z.g1_fixed_base(dev(k))
    got_dev = Z.msm_g1(pts, dev(sc))
    got_host = Z.msm_g1(Z.to_host(pts), sc)
    assert Z.msm_last_stats()["bucket_adds"] > 0
    assert np.array_equal(got_host, got_dev)
    exp = O.g1_fixed_base(O.fr_dot(k, sc)[None, :])[0]
    assert np.array_equal(got_dev, exp)


def test_g2_host_pipelined_matches_device():
    n = (1 << 20) + 5
    k = Z.random_fr(n, 51)
    sc = Z.random_fr(n, 52)
    pts = Z.g2_fixed_base(dev(k))
    got_dev = Z.msm_g2(pts, dev(sc))
    assert np.array_equal(Z.msm_g2(Z.to_host(pts), sc), got_dev)
    exp = O.g2_fixed_base(O.fr_dot(k, sc)[None, :])[0]
    assert np.array_equal(got_dev, exp)


@pytest.mark.parametrize("n", [129, 1000, 1 << 12])
def test_g2_matches_oracle(n):
    _, pts, sc = _random_instance(n, 300 + n, g2=True)
    exp = O.msm_g2(Z.to_host(pts), sc, nthreads=os.cpu_count())
    assert np.array_equal(Z.msm_g2(pts, dev(sc)), exp)


def test_g2_full_size_identity():
    n = 1 << 18
    k = Z.random_fr(n, 41)
    sc = Z.random_fr(n, 42)
    pts = Z.g2_fixed_base(dev(k))
    got = Z.msm_g2(pts, dev(sc))
    exp = O.g2_fixed_base(O.fr_dot(k, sc)[None, :])[0]
    assert np.array_equal(got, exp)


@pytest.mark.parametrize("scalars", ["uniform", "witness"])
def test_g2_witness_size_identity(scalars):
    """The G2 (B) MSM at config 5's witness size, 4,030,486 points, with
    uniform scalars and with a witness-like mix (69 % zero, 26 % one, the
    rest spread over small and full-width values): the identity
    sum_i s_i (k_i G2) = (sum_i s_i k_i) G2."""
    n = 4030486
    k = Z.random_fr(n, 61)
    sc = Z.random_fr(n, 62)
    if scalars == "witness":
        rng = np.random.default_rng(63)
        u = rng.random(n)
        sc[u < 0.69] = 0
        ones = (u >= 0.69) & (u < 0.95)
        sc[ones] = Z.fr_from_int(1)
        small = np.flatnonzero((u >= 0.95) & (u < 0.99))
        sc[small] = 0
        sc[small, 0] = rng.integers(2, 1 << 20, small.size).astype(np.uint64)
        sc[small] = O.fr_from_std_vector(sc[small])
    pts = Z.g2_fixed_base(dev(k))
    got = Z.msm_g2(pts, dev(sc))
    exp = O.g2_fixed_base(O.fr_dot(k, sc)[None, :])[0]
    assert np.array_equal(got, exp)


def _signed_scalars(n, seed):
    """Scalars of a signed witness: the folding boundary (r - 1) / 2 and
    (r + 1) / 2, r - 1, r - 2^k, then small positives and their negatives
    r - v, zeros and ones."""
    rng = np.random.default_rng(seed)
    vals = [0, 1, (O.R - 1) // 2, (O.R + 1) // 2, (O.R - 1) // 2 - 1, (O.R + 1) // 2 + 1, O.R - 1, O.R - 2]
    vals += [O.R - (1 << k) for k in (1, 31, 32, 63, 64, 128, 200, 252)]
    while len(vals) < n:
        v = int(rng.integers(1, 1 << 40))
        vals.append(v if rng.random() < 0.5 else O.R - v)
    return np.stack([O.fr_from_int(v) for v in vals[:n]])


@pytest.mark.parametrize("g2", [False, True])
def test_negative_scalars_fold(g2):
    """Scalars above (r - 1) / 2 are processed as r - s against -P (the same
    point): the boundary values and a signed witness match the oracle, and a
    witness of small magnitudes needs only the windows of its magnitudes."""
    n = 3000
    _, pts, _ = _random_instance(n, 0xF01D + g2, g2=g2)
    sc = _signed_scalars(n, 0xF01E)
    msm, omsm = (Z.msm_g2, O.msm_g2) if g2 else (Z.msm_g1, O.msm_g1)
    exp = omsm(Z.to_host(pts), sc, nthreads=os.cpu_count())
    assert np.array_equal(msm(pts, dev(sc)), exp)
    assert np.array_equal(msm(Z.to_host(pts), sc), exp)
    # magnitudes below 2^40 only: every scalar folds to at most 40 bits
    small = sc.copy()
    small[:16] = Z.fr_from_int(5)
    exp2 = omsm(Z.to_host(pts), small, nthreads=os.cpu_count())
    assert np.array_equal(msm(pts, dev(small)), exp2)
    st = Z.msm_last_stats()
    assert st["num_windows"] * st["window_bits"] <= 41 + st["window_bits"], st


def test_negative_scalars_fold_host_pipelined():
    """2^20 + 9 scalars, 30 % of them negative (r - v, v < 2^24), through the
    pipelined host path (its plan from the first batch's sample, all windows
    kept) and the device path, against the identity.  The witness MSMs of a
    proof (one shared sort) see such scalars in every prove test."""
    n = (1 << 20) + 9
    k = Z.random_fr(n, 0xF020)
    sc = Z.random_fr(n, 0xF021)
    rng = np.random.default_rng(0xF022)
    neg = np.flatnonzero(rng.random(n) < 0.3)
    mags = rng.integers(1, 1 << 24, neg.size)
    sc[neg] = np.stack([O.fr_from_int(O.R - int(v)) for v in mags])
    pts = Z.g1_fixed_base(dev(k))
    exp = O.g1_fixed_base(O.fr_dot(k, sc)[None, :])[0]
    assert np.array_equal(Z.msm_g1(pts, dev(sc)), exp)
    assert np.array_equal(Z.msm_g1(Z.to_host(pts), sc), exp)


def test_stats_and_probe():
    _, pts, sc = _random_instance(4096, 3)
    Z.msm_g1(pts, dev(sc))
    st = Z.msm_last_stats()
    assert st["kernel_launches"] >= 8 and st["accumulate_ms"] > 0
    assert Z.probe_imad_rate(0) > 1e12


@pytest.mark.parametrize("mode", ["1", "0"])
def test_g1_batch_affine_rounds_on_edge_cases(mode, monkeypatch):
    """The batch-affine rounds of the G1 accumulation (pairwise affine additions
    sharing one inversion per round) forced on (1) and off (0) for every case:
    the golden vectors (zero scalars, points at infinity, duplicates, P and -P,
    r - 1, all-zero inputs), a skewed mix with repeated points and opposite
    points in one bucket, and the oracle at several sizes."""
    monkeypatch.setenv("ZK_MSM_BATCH_AFFINE", mode)
    gz = g("g1_msm.npz")
    for name in cases(gz):
        pts, sc, res = gz[name + "_points"], gz[name + "_scalars"], gz[name + "_result"]
        assert np.array_equal(Z.msm_g1(dev(pts), dev(sc)), res), name
    n = 5000
    k, pts, sc = _random_instance(n, 0xBA00)
    ph = Z.to_host(pts)
    ph[100:200] = ph[300:400]                 # repeated points with repeated scalars: doublings
    sc[100:200] = sc[300:400]
    for i in range(500, 600):                 # -P beside P with the same scalar: P + (-P) in one bucket
        ph[i] = ph[i + 100]
        y = (O.P - O.to_int(ph[i + 100][4:8])) % O.P
        ph[i][4:8] = [(y >> (64 * w)) & (2**64 - 1) for w in range(4)]
    sc[500:600] = sc[600:700]
    ph[800:900] = 0                           # points at infinity
    sc[900:1000] = sc[7]                      # one hot bucket
    exp = O.msm_g1(ph, sc, nthreads=os.cpu_count())
    assert np.array_equal(Z.msm_g1(dev(ph), dev(sc)), exp)
    for n in (1, 2, 3, 255, 4097, 1 << 14):
        _, p2, s2 = _random_instance(n, 0xBA10 + n)
        assert np.array_equal(Z.msm_g1(p2, dev(s2)), O.msm_g1(Z.to_host(p2), s2, nthreads=os.cpu_count())), n


def test_g1_batch_affine_matches_serial_at_2_22(monkeypatch):
    """2^22 uniform points: the batch-affine rounds followed by the XYZZ
    accumulation of what they leave (ZK_MSM_BATCH_AFFINE=1) equal the default
    serial XYZZ accumulation and the identity sum k_i s_i G."""
    n = 1 << 22
    k = Z.random_fr(n, 0xBA22)
    sc = Z.random_fr(n, 0xBA23)
    pts = Z.g1_fixed_base(dev(k))
    exp = O.g1_fixed_base(O.fr_dot(k, sc)[None, :])[0]
    monkeypatch.setenv("ZK_MSM_BATCH_AFFINE", "1")
    assert np.array_equal(Z.msm_g1(pts, dev(sc)), exp)
    st = Z.msm_last_stats()
    assert st["batch_affine_pairs"] > n  # the rounds ran
    monkeypatch.delenv("ZK_MSM_BATCH_AFFINE")
    assert np.array_equal(Z.msm_g1(pts, dev(sc)), exp)
    assert Z.msm_last_stats()["batch_affine_pairs"] == 0
