"""ctypes binding for the CPU parity checker (oracle/liboracle.so) and, when it
was built here, the reference's own host arithmetic (oracle/_ref/libzkref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference legs of bench.py.  The product library never uses it.

Arrays are numpy uint64 with 4 limbs per field element (Montgomery form):
  Fr/Fp vectors  : shape (n, 4)
  G1 points      : shape (n, 8)  = x[4], y[4]; an all-zero row is infinity
  G2 points      : shape (n, 16) = x.c0, x.c1, y.c0, y.c1
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(HERE, "liboracle.so")
_REFLIB = os.path.join(HERE, "_ref", "libzkref.so")

_u64p = ctypes.POINTER(ctypes.c_uint64)


def reference_tree():
    """The reference checkout: $REF, else a directory named `reference` beside
    this repository (absent on machines that only run the prebuilt checkers)."""
    return os.environ.get("REF") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")


def build():
    """Compile liboracle.so (and _ref/ when the reference tree is present)."""
    targets = ["liboracle.so"]
    if os.path.isdir(reference_tree()):
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE] + targets, check=True)


def _load():
    if not os.path.exists(_LIB):
        subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    return ctypes.CDLL(_LIB)


lib = _load()


def ref_available():
    return os.path.exists(_REFLIB)


_ref = None


def ref():
    global _ref
    if _ref is None:
        _ref = ctypes.CDLL(_REFLIB)
    return _ref


def _p(a):
    assert a.dtype == np.uint64 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_u64p)


def u64(x, n=4):
    return np.array([(x >> (64 * i)) & ((1 << 64) - 1) for i in range(n)], dtype=np.uint64)


def to_int(limbs):
    return sum(int(v) << (64 * i) for i, v in enumerate(np.asarray(limbs).ravel()))


P = 21888242871839275222246405745257275088696311157297823662689037894645226208583
R = 21888242871839275222246405745257275088548364400416034343698204186575808495617


class Rng:
    """std::mt19937_64 stream (oracle/bn254_oracle.c orc_rng)."""

    class _S(ctypes.Structure):
        _fields_ = [("mt", ctypes.c_uint64 * 312), ("idx", ctypes.c_int)]

    def __init__(self, seed):
        self.s = Rng._S()
        lib.orc_rng_seed(ctypes.byref(self.s), ctypes.c_uint64(seed))
        lib.orc_rng_next.restype = ctypes.c_uint64

    def next(self):
        return lib.orc_rng_next(ctypes.byref(self.s))

    def fr_vector(self, n):
        out = np.zeros((n, 4), dtype=np.uint64)
        lib.orc_rand_fr_vec(ctypes.byref(self.s), _p(out), ctypes.c_size_t(n))
        return out


# ---------------------------------------------------------------- field
def fr_mul(a, b):
    o = np.zeros(4, dtype=np.uint64)
    lib.orc_fr_mul(_p(o), _p(np.ascontiguousarray(a, np.uint64)), _p(np.ascontiguousarray(b, np.uint64)))
    return o


def fp_mul(a, b):
    o = np.zeros(4, dtype=np.uint64)
    lib.orc_fp_mul(_p(o), _p(np.ascontiguousarray(a, np.uint64)), _p(np.ascontiguousarray(b, np.uint64)))
    return o


def fr_from_std_vector(a):
    """(n, 4) standard-form values below r -> Montgomery form."""
    a = np.ascontiguousarray(a, np.uint64).reshape(-1, 4)
    out = np.zeros_like(a)
    lib.orc_fr_from_std_vec(_p(out), _p(a), ctypes.c_size_t(a.shape[0]))
    return out


def fr_from_int(x):
    o = np.zeros(4, dtype=np.uint64)
    lib.orc_fr_from_std(_p(o), _p(u64(x % R)))
    return o


def fp_from_int(x):
    o = np.zeros(4, dtype=np.uint64)
    lib.orc_fp_from_std(_p(o), _p(u64(x % P)))
    return o


def fr_to_int(a):
    o = np.zeros(4, dtype=np.uint64)
    lib.orc_fr_to_std(_p(o), _p(np.ascontiguousarray(a, np.uint64)))
    return to_int(o)


def fp_to_int(a):
    o = np.zeros(4, dtype=np.uint64)
    lib.orc_fp_to_std(_p(o), _p(np.ascontiguousarray(a, np.uint64)))
    return to_int(o)


def compute_omega(log_n, inverse=False):
    o = np.zeros(4, dtype=np.uint64)
    lib.orc_compute_omega(_p(o), ctypes.c_int(log_n), ctypes.c_int(int(inverse)))
    return o


# ---------------------------------------------------------------- curves
class _G1A(ctypes.Structure):
    _fields_ = [("x", ctypes.c_uint64 * 4), ("y", ctypes.c_uint64 * 4), ("inf", ctypes.c_int)]


class _G2A(ctypes.Structure):
    _fields_ = [("v", ctypes.c_uint64 * 16), ("inf", ctypes.c_int)]


def _g1_out(s):
    if s.inf:
        return np.zeros(8, dtype=np.uint64)
    return np.array(list(s.x) + list(s.y), dtype=np.uint64)


def _g2_out(s):
    if s.inf:
        return np.zeros(16, dtype=np.uint64)
    return np.array(list(s.v), dtype=np.uint64)


def g1_generator():
    s = _G1A()
    lib.orc_g1_generator(ctypes.byref(s))
    return _g1_out(s)


def g2_generator():
    s = _G2A()
    lib.orc_g2_generator(ctypes.byref(s))
    return _g2_out(s)


def g1_fixed_base(scalars):
    """k_i * G1 for a (n, 4) Montgomery scalar array; returns (n, 8)."""
    scalars = np.ascontiguousarray(scalars, np.uint64)
    out = np.zeros((scalars.shape[0], 8), dtype=np.uint64)
    lib.orc_g1_fixed_base(_p(out), _p(scalars), ctypes.c_size_t(scalars.shape[0]), ctypes.c_int(os.cpu_count() or 1))
    return out


def g2_fixed_base(scalars):
    scalars = np.ascontiguousarray(scalars, np.uint64)
    out = np.zeros((scalars.shape[0], 16), dtype=np.uint64)
    lib.orc_g2_fixed_base(_p(out), _p(scalars), ctypes.c_size_t(scalars.shape[0]), ctypes.c_int(os.cpu_count() or 1))
    return out


def msm_g1(points, scalars, nthreads=1):
    points = np.ascontiguousarray(points, np.uint64)
    scalars = np.ascontiguousarray(scalars, np.uint64)
    s = _G1A()
    lib.orc_msm_g1(ctypes.byref(s), _p(points), _p(scalars), ctypes.c_size_t(scalars.shape[0]), ctypes.c_int(nthreads))
    return _g1_out(s)


def msm_g1_naive(points, scalars):
    points = np.ascontiguousarray(points, np.uint64)
    scalars = np.ascontiguousarray(scalars, np.uint64)
    s = _G1A()
    lib.orc_msm_g1_naive(ctypes.byref(s), _p(points), _p(scalars), ctypes.c_size_t(scalars.shape[0]))
    return _g1_out(s)


def msm_g2(points, scalars, nthreads=1):
    points = np.ascontiguousarray(points, np.uint64)
    scalars = np.ascontiguousarray(scalars, np.uint64)
    s = _G2A()
    lib.orc_msm_g2(ctypes.byref(s), _p(points), _p(scalars), ctypes.c_size_t(scalars.shape[0]), ctypes.c_int(nthreads))
    return _g2_out(s)


def msm_g2_naive(points, scalars):
    points = np.ascontiguousarray(points, np.uint64)
    scalars = np.ascontiguousarray(scalars, np.uint64)
    s = _G2A()
    lib.orc_msm_g2_naive(ctypes.byref(s), _p(points), _p(scalars), ctypes.c_size_t(scalars.shape[0]))
    return _g2_out(s)


def g1_on_curve(pt):
    s = _G1A()
    pt = np.asarray(pt, np.uint64)
    s.inf = int(not pt.any())
    for i in range(4):
        s.x[i] = int(pt[i]); s.y[i] = int(pt[4 + i])
    return bool(lib.orc_g1_is_on_curve(ctypes.byref(s)))


def g2_on_curve(pt):
    pt = np.ascontiguousarray(pt, np.uint64)
    return bool(lib.orc_g2_is_on_curve_raw(_p(pt)))


# ---------------------------------------------------------------- NTT
def ntt(a, log_n, inverse=False, nthreads=1):
    a = np.ascontiguousarray(a, np.uint64)
    out = np.zeros_like(a)
    lib.orc_ntt_mt(_p(out), _p(a), ctypes.c_int(log_n), ctypes.c_int(int(inverse)), ctypes.c_int(nthreads))
    return out


def ntt_naive(a, log_n, inverse=False):
    a = np.ascontiguousarray(a, np.uint64)
    out = np.zeros_like(a)
    lib.orc_ntt_naive(_p(out), _p(a), ctypes.c_int(log_n), ctypes.c_int(int(inverse)))
    return out


def coset_ntt(a, log_n, inverse, g, nthreads=1):
    a = np.ascontiguousarray(a, np.uint64)
    out = np.zeros_like(a)
    gg = np.ascontiguousarray(g, np.uint64)
    lib.orc_coset_ntt_mt(_p(out), _p(a), ctypes.c_int(log_n), ctypes.c_int(int(inverse)), _p(gg), ctypes.c_int(nthreads))
    return out


def compute_h_from_evals(a, b, c, log_n):
    a, b, c = (np.ascontiguousarray(x, np.uint64) for x in (a, b, c))
    out = np.zeros_like(a)
    lib.orc_compute_h_from_evals(_p(out), _p(a), _p(b), _p(c), ctypes.c_int(log_n))
    return out


def fr_dot(a, b, nthreads=None):
    a = np.ascontiguousarray(a, np.uint64)
    b = np.ascontiguousarray(b, np.uint64)
    o = np.zeros(4, dtype=np.uint64)
    lib.orc_fr_dot(_p(o), _p(a), _p(b), ctypes.c_size_t(a.shape[0]), ctypes.c_int(nthreads or os.cpu_count() or 1))
    return o


def fr_poly_eval(coeffs, x):
    coeffs = np.ascontiguousarray(coeffs, np.uint64)
    xx = np.ascontiguousarray(x, np.uint64)
    o = np.zeros(4, dtype=np.uint64)
    lib.orc_fr_poly_eval(_p(o), _p(coeffs), ctypes.c_size_t(coeffs.shape[0]), _p(xx))
    return o


def fr_pow(a, e):
    """a^e for a Montgomery Fr and a Python int e >= 0."""
    acc = fr_from_int(1)
    base = np.ascontiguousarray(a, np.uint64)
    while e:
        if e & 1:
            acc = fr_mul(acc, base)
        base = fr_mul(base, base)
        e >>= 1
    return acc
