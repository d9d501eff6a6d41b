"""Generate the committed golden vectors from the REFERENCE's own arithmetic.

Runs in a container where the reference tree exists: oracle/Makefile builds
oracle/_ref/libzkref.so from the reference's headers (src/field/fp.cuh,
src/field/fp2.cuh, src/curve/g1.cuh, src/curve/g2.cuh) and src/ntt/ntt.cu,
and this script drives it.  The outputs (small .npz files next to this
script) are what tests/ compare the oracle restatement and the CUDA library
against; nothing here is needed at test time.

Cases follow the reference's own tests where they exist:
  tests/test_msm.cu:40-127  (n=1: 5G; n=2: 3G+7G; n=64: i*G with scalars i+1;
                             G2 n=1: 5*G2; G2 n=16: i*G2 with scalars i+3)
  tests/test_ntt.cu:39-172  (n=4 input 1,2,3,4; round trips)
plus seeded random and edge cases (zero scalars, infinity points, duplicates,
P and -P, scalar r-1, small scalars).

    python tests/golden/make_golden.py
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import pyoracle  # noqa: E402

R = pyoracle.R
P = pyoracle.P
U64P = ctypes.POINTER(ctypes.c_uint64)


def p(a):
    return a.ctypes.data_as(U64P)


def main():
    pyoracle.build()
    if not pyoracle.ref_available():
        sys.exit("oracle/_ref/libzkref.so missing: the reference tree is needed to regenerate goldens")
    ref = pyoracle.ref()
    inf = ctypes.c_int()

    def rfr(x):
        o = np.zeros(4, np.uint64)
        ref.ref_fr_from_u64(p(o), ctypes.c_uint64(x))
        return o

    def fr_int(x):  # Montgomery form of a big integer, via the reference's from_standard for Fr
        x %= R
        return pyoracle.fr_from_int(x)

    def g1_smul(pt, k):
        o = np.zeros(8, np.uint64)
        ref.ref_g1_scalar_mul(p(o), ctypes.byref(inf), p(np.ascontiguousarray(pt)), int(not pt.any()), p(np.ascontiguousarray(k)))
        return o if not inf.value else np.zeros(8, np.uint64)

    def g2_smul(pt, k):
        o = np.zeros(16, np.uint64)
        ref.ref_g2_scalar_mul(p(o), ctypes.byref(inf), p(np.ascontiguousarray(pt)), int(not pt.any()), p(np.ascontiguousarray(k)))
        return o if not inf.value else np.zeros(16, np.uint64)

    def msm1(pts, sc):
        o = np.zeros(8, np.uint64)
        ref.ref_msm_g1_naive(p(o), ctypes.byref(inf), p(pts), p(sc), pts.shape[0])
        return o if not inf.value else np.zeros(8, np.uint64)

    def msm2(pts, sc):
        o = np.zeros(16, np.uint64)
        ref.ref_msm_g2_naive(p(o), ctypes.byref(inf), p(pts), p(sc), pts.shape[0])
        return o if not inf.value else np.zeros(16, np.uint64)

    rng = pyoracle.Rng(0x5EED0001)
    g1 = np.zeros(8, np.uint64)
    ref.ref_g1_generator(p(g1), ctypes.byref(inf))
    g2 = np.zeros(16, np.uint64)
    ref.ref_g2_generator(p(g2), ctypes.byref(inf))

    # ---------------------------------------------------------------- field
    a = rng.fr_vector(128)
    b = rng.fr_vector(128)
    out = {k: np.zeros((128, 4), np.uint64) for k in ("fr_mul", "fp_mul", "fr_add", "fr_sub", "fp_add", "fp_sub")}
    for i in range(128):
        ai, bi = np.ascontiguousarray(a[i]), np.ascontiguousarray(b[i])
        for k, fn in (("fr_mul", ref.ref_fr_mul), ("fp_mul", ref.ref_fp_mul), ("fr_add", ref.ref_fr_add),
                      ("fr_sub", ref.ref_fr_sub), ("fp_add", ref.ref_fp_add), ("fp_sub", ref.ref_fp_sub)):
            o = np.zeros(4, np.uint64)
            fn(p(o), p(ai), p(bi))
            out[k][i] = o
    fr_one = np.zeros(4, np.uint64)
    ref.ref_fr_one(p(fr_one))
    fp_one = np.zeros(4, np.uint64)
    ref.ref_fp_one(p(fp_one))
    np.savez(os.path.join(HERE, "field.npz"), a=a, b=b, fr_one=fr_one, fp_one=fp_one, **out)

    # ---------------------------------------------------------------- omega
    fwd = np.zeros((29, 4), np.uint64)
    inv = np.zeros((29, 4), np.uint64)
    for ln in range(29):
        o = np.zeros(4, np.uint64)
        ref.ref_compute_omega(p(o), ln, 0)
        fwd[ln] = o
        ref.ref_compute_omega(p(o), ln, 1)
        inv[ln] = o
    np.savez(os.path.join(HERE, "omega.npz"), fwd=fwd, inv=inv)

    # ---------------------------------------------------------------- G1 MSM
    cases = {}
    cases["n1"] = (g1[None, :].copy(), rfr(5)[None, :].copy())
    cases["n2"] = (np.stack([g1, g1]), np.stack([rfr(3), rfr(7)]))
    pts = np.stack([g1_smul(g1, rfr(i + 1)) for i in range(64)])
    cases["n64"] = (pts, np.stack([rfr(i + 1) for i in range(64)]))
    k = rng.fr_vector(257)
    pts = np.stack([g1_smul(g1, k[i]) for i in range(257)])
    cases["rand257"] = (pts, rng.fr_vector(257))
    # edge cases
    k = rng.fr_vector(48)
    pts = np.stack([g1_smul(g1, k[i]) for i in range(48)])
    sc = rng.fr_vector(48)
    pts[3] = 0                     # infinity point with a nonzero scalar
    pts[7] = 0
    sc[5] = 0                      # zero scalars
    sc[6] = 0
    pts[10] = pts[11]              # duplicate points
    sc[10] = sc[11]                # same point, same scalar -> bucket doubling
    neg = pts[12].copy()           # P and -P
    yint = pyoracle.fp_to_int(neg[4:8])
    neg[4:8] = pyoracle.fp_from_int((P - yint) % P)
    pts[13] = neg
    sc[13] = sc[12]
    sc[14] = fr_int(R - 1)         # scalar r - 1
    sc[15] = rfr(1)
    sc[16] = rfr(0xFFFF)           # small scalars
    sc[17] = rfr(1 << 15)
    sc[18] = fr_int((1 << 253) + 12345)
    cases["edge48"] = (pts, sc)
    cases["all_zero_scalars"] = (pts[:20].copy(), np.zeros((20, 4), np.uint64))
    cases["all_infinity"] = (np.zeros((9, 8), np.uint64), rng.fr_vector(9))
    cases["pm_cancel"] = (np.stack([pts[12], neg]), np.stack([sc[12], sc[12]]))
    small = np.stack([rfr(int(rng.next() & 0xFFFF)) for _ in range(100)])
    cases["small100"] = (cases["rand257"][0][:100].copy(), small)
    g1_out = {}
    for name, (pts_, sc_) in cases.items():
        pts_ = np.ascontiguousarray(pts_, np.uint64)
        sc_ = np.ascontiguousarray(sc_, np.uint64)
        g1_out[name + "_points"] = pts_
        g1_out[name + "_scalars"] = sc_
        g1_out[name + "_result"] = msm1(pts_, sc_)
    np.savez(os.path.join(HERE, "g1_msm.npz"), **g1_out)

    # ---------------------------------------------------------------- G2 MSM
    c2 = {}
    c2["n1"] = (g2[None, :].copy(), rfr(5)[None, :].copy())
    pts2 = np.stack([g2_smul(g2, rfr(i + 1)) for i in range(16)])
    c2["n16"] = (pts2, np.stack([rfr(i + 3) for i in range(16)]))
    k = rng.fr_vector(12)
    pts2 = np.stack([g2_smul(g2, k[i]) for i in range(12)])
    sc2 = rng.fr_vector(12)
    pts2[4] = 0
    sc2[6] = 0
    sc2[7] = fr_int(R - 1)
    c2["edge12"] = (pts2, sc2)
    g2_out = {}
    for name, (pts_, sc_) in c2.items():
        pts_ = np.ascontiguousarray(pts_, np.uint64)
        sc_ = np.ascontiguousarray(sc_, np.uint64)
        g2_out[name + "_points"] = pts_
        g2_out[name + "_scalars"] = sc_
        g2_out[name + "_result"] = msm2(pts_, sc_)
    np.savez(os.path.join(HERE, "g2_msm.npz"), **g2_out)

    # ---------------------------------------------------------------- NTT
    ntt_out = {}
    x = np.stack([rfr(v) for v in (1, 2, 3, 4)])
    for name, arr, ln in [("n4_1234", x, 2)] + [(f"rand_log{ln}", rng.fr_vector(1 << ln), ln) for ln in (0, 1, 2, 3, 4, 5, 7, 8, 10)]:
        arr = np.ascontiguousarray(arr, np.uint64)
        f = np.zeros_like(arr)
        ref.ref_ntt_naive(p(f), p(arr), ln, 0)
        iv = np.zeros_like(arr)
        ref.ref_ntt_naive(p(iv), p(arr), ln, 1)
        ntt_out[name + "_in"] = arr
        ntt_out[name + "_fwd"] = f
        ntt_out[name + "_inv"] = iv
        ntt_out[name + "_log"] = np.array([ln])
    np.savez(os.path.join(HERE, "ntt.npz"), **ntt_out)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
