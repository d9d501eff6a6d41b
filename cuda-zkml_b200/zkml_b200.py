"""Python binding of libzkml_b200.so (ctypes over the C ABI in include/zkml_b200.h).

Device buffers are torch CUDA tensors (any dtype; the raw bytes are used) and
calls are ordered on torch's current CUDA stream.  Host buffers are numpy
arrays.  Field elements are 32-byte Montgomery-form little-endian values:
numpy uint64 arrays of shape (n, 4); packed G1 points are (n, 8), packed G2
points (n, 16); the all-zero record is the point at infinity.

There is no CPU fallback: if the shared library is missing this module raises
at import, and every compute call raises ZkError when no CUDA device is usable.
"""
import ctypes
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("ZKML_B200_LIB", os.path.join(HERE, "libzkml_b200.so"))
HEADER = os.path.join(os.path.dirname(HERE), "include", "zkml_b200.h")

ZK_OK, ZK_ERR_INVALID, ZK_ERR_CUDA, ZK_ERR_NOMEM, ZK_ERR_NODEV, ZK_ERR_RANGE = 0, 1, 2, 3, 4, 5

R_MOD = 21888242871839275222246405745257275088548364400416034343698204186575808495617
P_MOD = 21888242871839275222246405745257275088696311157297823662689037894645226208583


class ZkError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"zkml_b200 status {status}: {message}")
        self.status = status


if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is not built (run `make -C {HERE}` or __graft_entry__.build())")

lib = ctypes.CDLL(LIB_PATH)
lib.zk_last_error.restype = ctypes.c_char_p
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_i = ctypes.c_int


class MsmStats(ctypes.Structure):
    _fields_ = [("kernel_launches", ctypes.c_int), ("accumulate_ms", ctypes.c_float),
                ("total_device_ms", ctypes.c_float), ("window_bits", ctypes.c_int),
                ("num_windows", ctypes.c_int), ("bucket_adds", ctypes.c_longlong),
                ("phase_ms", ctypes.c_float * 8), ("batch_affine_pairs", ctypes.c_longlong),
                ("batch_affine_left", ctypes.c_longlong)]


class Groth16Arrays(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("m", ctypes.c_int), ("num_public", ctypes.c_int), ("l", ctypes.c_int),
                ("n_h", ctypes.c_int), ("a", _vp), ("b1", _vp), ("b2", _vp), ("l_query", _vp), ("h_query", _vp)]


_SIGS = {
    "zk_device_count": [ctypes.POINTER(ctypes.c_int)],
    "zk_version": [],
    "zk_msm_g1": [_vp, _vp, _i, _vp],
    "zk_msm_g2": [_vp, _vp, _i, _vp],
    "zk_ntt": [_vp, _vp, _i, _i],
    "zk_ntt_inplace": [_vp, _i, _i],
    "zk_compute_omega": [_i, _i, _vp],
    "zk_msm_g1_device": [_i, _vp, _vp, _vp, _sz, _vp],
    "zk_msm_g1_host": [_i, _vp, _vp, _vp, _sz, _vp],
    "zk_msm_g2_device": [_i, _vp, _vp, _vp, _sz, _vp],
    "zk_msm_g2_host": [_i, _vp, _vp, _vp, _sz, _vp],
    "zk_ntt_device": [_i, _vp, _vp, _vp, _i, _i, _vp],
    "zk_compute_h_device": [_i, _vp, _vp, _vp, _vp, _vp, _i],
    "zk_g1_fixed_base_device": [_i, _vp, _vp, _vp, _sz],
    "zk_g2_fixed_base_device": [_i, _vp, _vp, _vp, _sz],
    "zk_g1_add_affine": [_vp, _vp, _vp],
    "zk_g2_add_affine": [_vp, _vp, _vp],
    "zk_probe_imad_rate": [_i, ctypes.POINTER(ctypes.c_double)],
    "zk_msm_last_stats": [ctypes.POINTER(MsmStats)],
    "zk_r1cs_matvec_rows_device": [_vp, _vp, _vp, ctypes.c_uint64, ctypes.c_uint64, _vp],
    "zk_fr_hadamard_check_device": [_i, _vp, _vp, _vp, _vp, _sz, ctypes.c_uint64, ctypes.POINTER(ctypes.c_longlong)],
    "zk_compute_h_coset_shift": [_i, _vp],
    "zk_compute_h_pointwise_device": [_i, _vp, _vp, _vp, _vp, _vp, _i, ctypes.c_uint64],
    "zk_ntt_cross_device": [_i, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _i],
    "zk_groth16_pk_arrays": [_vp, ctypes.POINTER(Groth16Arrays)],
    "zk_groth16_assemble": [_vp, _vp, _vp, _vp, _vp, _vp],
    "zk_groth16_assemble_parts": [_vp, _vp, _vp, _vp, _i, _vp, _vp],
    "zk_groth16_h_msm_device": [_vp, _vp, _vp, ctypes.c_uint64, ctypes.c_uint64, _vp],
    "zk_groth16_h_msm_blocks_device": [_vp, _vp, _vp, _i, _i, _vp],
    "zk_groth16_precompute": [_vp, _vp],
    "zk_groth16_witness_msms_device": [_vp, _vp, _vp, ctypes.c_uint64, ctypes.c_uint64, _vp],
}
for _name, _args in _SIGS.items():
    getattr(lib, _name).argtypes = _args
    getattr(lib, _name).restype = ctypes.c_int


def declared_symbols():
    """Function names declared in include/zkml_b200.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*|void)\s+(zk_\w+)\s*\(", text, re.M)))


def check(status):
    if status != ZK_OK:
        raise ZkError(status, lib.zk_last_error().decode(errors="replace"))


def last_error():
    return lib.zk_last_error().decode(errors="replace")


def device_count():
    c = ctypes.c_int(0)
    check(lib.zk_device_count(ctypes.byref(c)))
    return c.value


# ------------------------------------------------------------------ helpers
def _np_ptr(a):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_vp)


def _torch():
    import torch
    return torch


def _dev_ptr(t):
    torch = _torch()
    assert isinstance(t, torch.Tensor) and t.is_cuda and t.is_contiguous(), "expected a contiguous CUDA tensor"
    return ctypes.c_void_p(t.data_ptr())


def _stream(t):
    torch = _torch()
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def to_device(arr, device="cuda"):
    """numpy uint64 array -> int64 CUDA tensor with the same bytes."""
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int64)).to(device)


def to_host(t):
    """CUDA tensor -> numpy uint64 array with the same bytes."""
    return t.detach().cpu().numpy().view(np.uint64)


def random_fr(n, seed):
    """n uniform Fr values (Montgomery form is a bijection of [0, r), so uniform
    canonical values are uniform Montgomery representations): (n, 4) uint64."""
    rng = np.random.default_rng(seed)
    out = np.empty((n, 4), dtype=np.uint64)
    need = np.arange(n)
    r_top = R_MOD >> 192
    while need.size:
        cand = rng.integers(0, 2**64, size=(need.size, 4), dtype=np.uint64)
        cand[:, 3] &= np.uint64((1 << 62) - 1)
        top = cand[:, 3]
        ok = top < np.uint64(r_top)  # strictly below r's top limb => below r
        out[need[ok]] = cand[ok]
        need = need[~ok]
    return out


def fr_from_int(x):
    """Montgomery form of the integer x mod r as (4,) uint64."""
    v = (x % R_MOD) * (1 << 256) % R_MOD
    return np.array([(v >> (64 * i)) & (2**64 - 1) for i in range(4)], dtype=np.uint64)


def fr_to_int(limbs):
    v = sum(int(w) << (64 * i) for i, w in enumerate(np.asarray(limbs, dtype=np.uint64).ravel()))
    return v * pow(1 << 256, -1, R_MOD) % R_MOD


# ------------------------------------------------------------------ MSM
def msm_g1(points, scalars, device=None):
    """Sum s_i P_i over G1.  torch CUDA tensors -> device path on the current
    stream; numpy arrays -> host path (copies pipelined inside).  Returns the
    affine result as (8,) uint64 (all zero for the identity)."""
    return _msm(points, scalars, device, g2=False)


def msm_g2(points, scalars, device=None):
    return _msm(points, scalars, device, g2=True)


def _msm(points, scalars, device, g2):
    words = 16 if g2 else 8
    out = np.zeros(words, dtype=np.uint64)
    if isinstance(points, np.ndarray):
        points = np.ascontiguousarray(points, dtype=np.uint64)
        scalars = np.ascontiguousarray(scalars, dtype=np.uint64)
        n = scalars.shape[0]
        fn = lib.zk_msm_g2_host if g2 else lib.zk_msm_g1_host
        check(fn(-1 if device is None else device, None, _np_ptr(points), _np_ptr(scalars), n, _np_ptr(out)))
    else:
        n = scalars.numel() * scalars.element_size() // 32
        dev = points.device.index if device is None else device
        fn = lib.zk_msm_g2_device if g2 else lib.zk_msm_g1_device
        check(fn(dev, _stream(points), _dev_ptr(points), _dev_ptr(scalars), n, _np_ptr(out)))
    return out


def msm_g1_ref(points72, scalars, n=None):
    """Reference-shaped msm_g1: 72-byte host records (uint8 array), host Fr;
    returns the 96-byte G1Jacobian as (12,) uint64."""
    points72 = np.ascontiguousarray(points72, dtype=np.uint8)
    scalars = np.ascontiguousarray(scalars, dtype=np.uint64)
    n = scalars.shape[0] if n is None else n
    out = np.zeros(12, dtype=np.uint64)
    check(lib.zk_msm_g1(_np_ptr(points72), _np_ptr(scalars), n, _np_ptr(out)))
    return out


def msm_g2_ref(points136, scalars, n=None):
    points136 = np.ascontiguousarray(points136, dtype=np.uint8)
    scalars = np.ascontiguousarray(scalars, dtype=np.uint64)
    n = scalars.shape[0] if n is None else n
    out = np.zeros(24, dtype=np.uint64)
    check(lib.zk_msm_g2(_np_ptr(points136), _np_ptr(scalars), n, _np_ptr(out)))
    return out


def packed_to_ref_g1(points):
    """(n, 8) packed -> (n, 72) uint8 reference G1Affine records."""
    points = np.ascontiguousarray(points, dtype=np.uint64)
    n = points.shape[0]
    rec = np.zeros((n, 9), dtype=np.uint64)
    rec[:, :8] = points
    rec[:, 8] = (~points.any(axis=1)).astype(np.uint64)
    return rec.view(np.uint8).reshape(n, 72)


def packed_to_ref_g2(points):
    points = np.ascontiguousarray(points, dtype=np.uint64)
    n = points.shape[0]
    rec = np.zeros((n, 17), dtype=np.uint64)
    rec[:, :16] = points
    rec[:, 16] = (~points.any(axis=1)).astype(np.uint64)
    return rec.view(np.uint8).reshape(n, 136)


def msm_last_stats():
    s = MsmStats()
    check(lib.zk_msm_last_stats(ctypes.byref(s)))
    d = {k: getattr(s, k) for k, _ in MsmStats._fields_}
    d["phase_ms"] = dict(zip(MSM_PHASES, list(s.phase_ms)))
    return d


MSM_PHASES = ("count", "scan", "scatter", "accumulate", "fixup", "reduce", "windows", "result_copy")


def g1_fixed_base(scalars_dev, out=None):
    """k_i * G1 for Montgomery scalars on the device -> (n, 8) int64 CUDA tensor."""
    torch = _torch()
    n = scalars_dev.numel() * scalars_dev.element_size() // 32
    if out is None:
        out = torch.empty((n, 8), dtype=torch.int64, device=scalars_dev.device)
    check(lib.zk_g1_fixed_base_device(scalars_dev.device.index, _stream(scalars_dev), _dev_ptr(out), _dev_ptr(scalars_dev), n))
    return out


def g2_fixed_base(scalars_dev, out=None):
    torch = _torch()
    n = scalars_dev.numel() * scalars_dev.element_size() // 32
    if out is None:
        out = torch.empty((n, 16), dtype=torch.int64, device=scalars_dev.device)
    check(lib.zk_g2_fixed_base_device(scalars_dev.device.index, _stream(scalars_dev), _dev_ptr(out), _dev_ptr(scalars_dev), n))
    return out


def g1_add_affine(a, b):
    a = np.ascontiguousarray(a, dtype=np.uint64)
    b = np.ascontiguousarray(b, dtype=np.uint64)
    out = np.zeros(8, dtype=np.uint64)
    check(lib.zk_g1_add_affine(_np_ptr(a), _np_ptr(b), _np_ptr(out)))
    return out


def g2_add_affine(a, b):
    a = np.ascontiguousarray(a, dtype=np.uint64)
    b = np.ascontiguousarray(b, dtype=np.uint64)
    out = np.zeros(16, dtype=np.uint64)
    check(lib.zk_g2_add_affine(_np_ptr(a), _np_ptr(b), _np_ptr(out)))
    return out


# ------------------------------------------------------------------ NTT
def ntt(x, log_n, inverse=False, coset=None, out=None):
    """NTT of a CUDA tensor holding 2^log_n Fr values (natural order in/out).
    coset: None or a (4,) uint64 Montgomery Fr shift g."""
    torch = _torch()
    if out is None:
        out = torch.empty_like(x)
    g = None
    if coset is not None:
        gc = np.ascontiguousarray(coset, dtype=np.uint64)
        g = _np_ptr(gc)
    check(lib.zk_ntt_device(x.device.index, _stream(x), _dev_ptr(out), _dev_ptr(x), log_n, int(inverse), g))
    return out


def compute_h_coset_shift(log_n):
    """compute_h's coset shift g (Montgomery (4,) uint64): 5, or 7 when 5^n = 1."""
    g = np.zeros(4, np.uint64)
    check(lib.zk_compute_h_coset_shift(log_n, _np_ptr(g)))
    return g


def compute_h_pointwise(a, b, c, log_n, out=None):
    """(a b - c) / (g^n - 1) elementwise over coset evaluations of the 2^log_n
    domain (CUDA tensors: all of them, or one part's share)."""
    torch = _torch()
    if out is None:
        out = torch.empty_like(a)
    check(lib.zk_compute_h_pointwise_device(a.device.index, _stream(a), _dev_ptr(out), _dev_ptr(a), _dev_ptr(b), _dev_ptr(c),
                                            log_n, a.shape[0]))
    return out


def ntt_cross(x, log_n, log_parts, part, inverse, mode, factor=None, factor_inverse=False, out=None):
    """One part's cross-part step of a 2^log_n-point transform split over
    2^log_parts parts (zk_ntt_cross_device): mode 0 cyclic -> blocks (after the
    size-m transform and the all-to-all), mode 1 blocks -> cyclic (before them).
    factor: None or a (4,) uint64 Montgomery g, applied as g^i (g^-i with
    factor_inverse) at global index i."""
    torch = _torch()
    if out is None:
        out = torch.empty_like(x)
    g = None
    if factor is not None:
        gc = np.ascontiguousarray(factor, dtype=np.uint64)
        g = _np_ptr(gc)
    check(lib.zk_ntt_cross_device(x.device.index, _stream(x), _dev_ptr(out), _dev_ptr(x), log_n, log_parts, part, int(inverse),
                                  mode, g, int(factor_inverse)))
    return out


def hadamard_check(a, b, c, row0=0):
    """First row0 + i with a_i b_i != c_i, or -1 (CUDA tensors of equal length)."""
    bad = ctypes.c_longlong()
    count = a.numel() * a.element_size() // 32
    check(lib.zk_fr_hadamard_check_device(a.device.index, _stream(a), _dev_ptr(a), _dev_ptr(b), _dev_ptr(c), count, row0,
                                          ctypes.byref(bad)))
    return bad.value


def ntt_ref(d_out, d_in, log_n, inverse):
    """Reference-shaped ntt_gpu (synchronous, current device)."""
    return lib.zk_ntt(_dev_ptr(d_out), _dev_ptr(d_in), log_n, int(inverse))


def compute_h(a, b, c, log_n, out=None):
    torch = _torch()
    if out is None:
        out = torch.empty_like(a)
    check(lib.zk_compute_h_device(a.device.index, _stream(a), _dev_ptr(out), _dev_ptr(a), _dev_ptr(b), _dev_ptr(c), log_n))
    return out


def compute_omega(log_n, inverse=False):
    out = np.zeros(4, dtype=np.uint64)
    check(lib.zk_compute_omega(log_n, int(inverse), _np_ptr(out)))
    return out


def probe_imad_rate(device=0):
    r = ctypes.c_double(0)
    check(lib.zk_probe_imad_rate(device, ctypes.byref(r)))
    return r.value


class IntPipeRates(ctypes.Structure):
    _fields_ = [("mad_lo_per_s", ctypes.c_double), ("mad_hi_per_s", ctypes.c_double), ("mad_pair_per_s", ctypes.c_double),
                ("sm_clock_ghz", ctypes.c_double), ("mad_lo_per_clk_sm", ctypes.c_double),
                ("mad_hi_per_clk_sm", ctypes.c_double), ("mad_pair_per_clk_sm", ctypes.c_double), ("num_sms", ctypes.c_int)]


lib.zk_probe_int_pipe.argtypes = [ctypes.c_int, ctypes.POINTER(IntPipeRates)]


def probe_int_pipe(device=0):
    """Hardware issue rates of mad.lo / mad.hi / lo+hi pairs (instructions/s and
    per clock per SM at the SM clock the probe measured)."""
    r = IntPipeRates()
    check(lib.zk_probe_int_pipe(device, ctypes.byref(r)))
    return {f: getattr(r, f) for f, _ in IntPipeRates._fields_}


# ------------------------------------------------------------------ Groth16
ENTRY_DTYPE = np.dtype([("row", "<i4"), ("col", "<i4"), ("v", "<u8", (4,))])  # zkml::SparseEntry


class _Synth(ctypes.Structure):
    _fields_ = [("num_constraints", ctypes.c_int), ("num_variables", ctypes.c_int), ("num_public", ctypes.c_int),
                ("nnz", ctypes.c_size_t * 3), ("entries", ctypes.c_void_p * 3), ("witness", ctypes.c_void_p)]


class ProveStats(ctypes.Structure):
    _fields_ = [("matvec_ms", ctypes.c_float), ("compute_h_ms", ctypes.c_float), ("msm_ms", ctypes.c_float * 5),
                ("total_ms", ctypes.c_float)]


lib.zk_synth_conv_circuit.argtypes = [_i, _i, _i, _i, _i, _i, _i, _i, ctypes.c_uint64, ctypes.POINTER(_Synth)]
lib.zk_synth_conv_circuit.restype = _i
lib.zk_synth_mlp_circuit.argtypes = [_i, _i, _i, _i, _i, _i, _i, ctypes.c_uint64, ctypes.POINTER(_Synth)]
lib.zk_synth_mlp_circuit.restype = _i
lib.zk_synth_free.argtypes = [ctypes.POINTER(_Synth)]
lib.zk_synth_free.restype = None
lib.zk_r1cs_create.argtypes = [_i, _i, _i, _i, _vp, _sz, _vp, _sz, _vp, _sz, ctypes.POINTER(_vp)]
lib.zk_r1cs_create.restype = _i
lib.zk_r1cs_destroy.argtypes = [_vp]
lib.zk_r1cs_destroy.restype = None
lib.zk_r1cs_domain.argtypes = [_vp, ctypes.POINTER(ctypes.c_int)]
lib.zk_groth16_setup.argtypes = [_vp, _vp, ctypes.POINTER(_vp)]
lib.zk_groth16_pk_load.argtypes = [_i, ctypes.c_char_p, ctypes.POINTER(_vp)]
lib.zk_groth16_pk_save.argtypes = [_vp, ctypes.c_char_p]
lib.zk_groth16_vk_save.argtypes = [_vp, ctypes.c_char_p]
lib.zk_groth16_vk_points.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _i]
lib.zk_groth16_pk_destroy.argtypes = [_vp]
lib.zk_groth16_pk_destroy.restype = None
lib.zk_groth16_prove.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]
lib.zk_groth16_last_stats.argtypes = [ctypes.POINTER(ProveStats)]


def synth_conv_circuit(layers=2, channels=32, height=32, width=32, bits=24, shift=10, out_bits=23, dense=10, seed=5):
    """Seeded CONV/ReLU R1CS with a satisfying witness (host numpy copies)."""
    c = _Synth()
    check(lib.zk_synth_conv_circuit(layers, channels, height, width, bits, shift, out_bits, dense, seed, ctypes.byref(c)))
    return _synth_copy(c)


def synth_mlp_circuit(batch=4, n_in=64, n_hidden=32, n_out=10, bits=24, shift=6, context=True, seed=1):
    """Seeded MLP statement (LINEAR, RELU_EXACT, LINEAR over a batch, context-bound)
    with a satisfying witness (host numpy copies)."""
    c = _Synth()
    check(lib.zk_synth_mlp_circuit(batch, n_in, n_hidden, n_out, bits, shift, int(context), seed, ctypes.byref(c)))
    return _synth_copy(c)


def _synth_copy(c):
    try:
        mats = []
        for k in range(3):
            nbytes = 40 * c.nnz[k]
            raw = np.ctypeslib.as_array((ctypes.c_uint8 * max(nbytes, 1)).from_address(c.entries[k]))[:nbytes]
            mats.append(raw.copy().view(ENTRY_DTYPE))
        m = c.num_variables
        w = np.ctypeslib.as_array((ctypes.c_uint64 * (4 * m)).from_address(c.witness)).copy().reshape(m, 4)
        return {"A": mats[0], "B": mats[1], "C": mats[2], "witness": w, "num_constraints": c.num_constraints,
                "num_variables": m, "num_public": c.num_public}
    finally:
        lib.zk_synth_free(ctypes.byref(c))


class R1cs:
    """Constraint system resident on one device (zk_r1cs)."""

    def __init__(self, circuit, device=0):
        self.h = _vp()
        mats = [np.ascontiguousarray(circuit[k]) for k in "ABC"]
        check(lib.zk_r1cs_create(device, circuit["num_constraints"], circuit["num_variables"], circuit["num_public"],
                                 _np_ptr(mats[0]), len(mats[0]), _np_ptr(mats[1]), len(mats[1]),
                                 _np_ptr(mats[2]), len(mats[2]), ctypes.byref(self.h)))
        ln = ctypes.c_int()
        check(lib.zk_r1cs_domain(self.h, ctypes.byref(ln)))
        self.log_n = ln.value
        self.num_constraints = circuit["num_constraints"]
        self.num_variables = circuit["num_variables"]
        self.num_public = circuit["num_public"]

    def matvec_rows(self, d_witness, lo, hi, out=None):
        """Rows [lo, hi) of A w, B w, C w as a (3, hi - lo, 4) int64 CUDA tensor."""
        torch = _torch()
        if out is None:
            out = torch.empty((3, hi - lo, 4), dtype=torch.int64, device=d_witness.device)
        check(lib.zk_r1cs_matvec_rows_device(self.h, _stream(d_witness), _dev_ptr(d_witness), lo, hi,
                                             _dev_ptr(out) if hi > lo else None))
        return out

    def __del__(self):
        if getattr(self, "h", None):
            lib.zk_r1cs_destroy(self.h)
            self.h = None


class PkLoadStats(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_double), ("read_ms", ctypes.c_double), ("total_ms", ctypes.c_double),
                ("alloc_ms", ctypes.c_double)]


lib.zk_groth16_pk_last_load_stats.argtypes = [ctypes.POINTER(PkLoadStats)]


class ProvingKey:
    """Proving key resident on one device (zk_groth16_pk)."""

    def __init__(self, handle):
        self.h = handle

    @classmethod
    def setup(cls, r1cs, toxic):
        """toxic: (tau, alpha, beta, gamma, delta) as Python ints."""
        tx = np.stack([fr_from_int(t) for t in toxic])
        h = _vp()
        check(lib.zk_groth16_setup(r1cs.h, _np_ptr(tx), ctypes.byref(h)))
        return cls(h)

    @classmethod
    def load(cls, path, device=0):
        h = _vp()
        check(lib.zk_groth16_pk_load(device, path.encode(), ctypes.byref(h)))
        return cls(h)

    @staticmethod
    def last_load_stats():
        """Bytes of query records, host read time, whole-call time and
        allocation time of this thread's last load
        (zk_groth16_pk_last_load_stats)."""
        st = PkLoadStats()
        check(lib.zk_groth16_pk_last_load_stats(ctypes.byref(st)))
        return {"bytes": st.bytes, "read_ms": st.read_ms, "total_ms": st.total_ms, "alloc_ms": st.alloc_ms}

    def save(self, path):
        check(lib.zk_groth16_pk_save(self.h, path.encode()))

    def save_vk(self, path):
        check(lib.zk_groth16_vk_save(self.h, path.encode()))

    def vk_points(self):
        a1 = np.zeros(8, np.uint64)
        b2, g2, d2 = (np.zeros(16, np.uint64) for _ in range(3))
        nic = lib.zk_groth16_vk_points(self.h, None, None, None, None, None, 0)
        ic = np.zeros((max(nic, 1), 8), np.uint64)
        lib.zk_groth16_vk_points(self.h, _np_ptr(a1), _np_ptr(b2), _np_ptr(g2), _np_ptr(d2), _np_ptr(ic), nic)
        return {"alpha1": a1, "beta2": b2, "gamma2": g2, "delta2": d2, "ic": ic[:nic]}

    def arrays(self):
        """Device pointers and sizes of the query arrays (zk_groth16_pk_arrays)."""
        a = Groth16Arrays()
        check(lib.zk_groth16_pk_arrays(self.h, ctypes.byref(a)))
        return {k: getattr(a, k) for k, _ in Groth16Arrays._fields_}

    def assemble(self, r, s, sums):
        """Proof from the five MSM sums (A, B2, L, H, B1 packed affine; 48 words)."""
        rr, ss = fr_from_int(r), fr_from_int(s)
        sums = np.ascontiguousarray(sums, dtype=np.uint64)
        assert sums.size == 48
        proof = np.zeros(256, np.uint8)
        pts = np.zeros(32, np.uint64)
        check(lib.zk_groth16_assemble(self.h, _np_ptr(rr), _np_ptr(ss), _np_ptr(sums), _np_ptr(proof), _np_ptr(pts)))
        return proof.tobytes(), pts[:8], pts[8:24], pts[24:32]

    def precompute(self, stream=None):
        """Build the H-query window tables now and wait for them (else the
        first proof starts their build as it ends and proofs run without them
        until it is done)."""
        check(lib.zk_groth16_precompute(self.h, stream))

    def witness_msms(self, d_w, lo, hi):
        """A, B2, B1 and L sums over the witness slice [lo, hi) (d_w: the whole
        witness on the device), one shared sort: a 48-word sums record with H zero."""
        rec = np.zeros(48, np.uint64)
        check(lib.zk_groth16_witness_msms_device(self.h, _stream(d_w), _dev_ptr(d_w), lo, hi, _np_ptr(rec)))
        return rec

    def h_msm(self, d_h, lo, hi):
        """sum_{i in [lo, hi)} h_i H_i over the key's H query (d_h: all n_h
        coefficients on the device); packed affine (8,) uint64."""
        out = np.zeros(8, np.uint64)
        check(lib.zk_groth16_h_msm_device(self.h, _stream(d_h), _dev_ptr(d_h), lo, hi, _np_ptr(out)))
        return out

    def h_msm_blocks(self, d_h_part, log_parts, part):
        """This part's share of the H MSM of a proof split over 2^log_parts parts:
        its coefficients (CUDA tensor) in the "blocks" layout of ntt_cross."""
        out = np.zeros(8, np.uint64)
        check(lib.zk_groth16_h_msm_blocks_device(self.h, _stream(d_h_part), _dev_ptr(d_h_part), log_parts, part, _np_ptr(out)))
        return out

    def assemble_parts(self, r, s, parts):
        """Proof from per-rank partial sums (a list of 48-word records), summed first."""
        rr, ss = fr_from_int(r), fr_from_int(s)
        rec = np.ascontiguousarray(np.stack([np.asarray(p, dtype=np.uint64)[:48] for p in parts]))
        proof = np.zeros(256, np.uint8)
        pts = np.zeros(32, np.uint64)
        check(lib.zk_groth16_assemble_parts(self.h, _np_ptr(rr), _np_ptr(ss), _np_ptr(rec), len(parts), _np_ptr(proof),
                                            _np_ptr(pts)))
        return proof.tobytes(), pts[:8], pts[8:24], pts[24:32]

    def prove(self, r1cs, witness, r, s, stream=None):
        """witness (m, 4) Montgomery; r, s ints.  Returns (proof bytes, A, B, C)."""
        witness = np.ascontiguousarray(witness, dtype=np.uint64)
        rr, ss = fr_from_int(r), fr_from_int(s)
        proof = np.zeros(256, np.uint8)
        pts = np.zeros(32, np.uint64)
        check(lib.zk_groth16_prove(self.h, r1cs.h, stream, _np_ptr(witness), _np_ptr(rr), _np_ptr(ss), _np_ptr(proof), _np_ptr(pts)))
        return proof.tobytes(), pts[:8], pts[8:24], pts[24:32]

    def __del__(self):
        if getattr(self, "h", None):
            lib.zk_groth16_pk_destroy(self.h)
            self.h = None


# ------------------------------------------------------------------ split prove (C, several devices)
class SplitStats(ctypes.Structure):
    _fields_ = [("nranks", ctypes.c_int), ("rank", ctypes.c_int), ("witness_ms", ctypes.c_float), ("matvec_ms", ctypes.c_float),
                ("compute_h_ms", ctypes.c_float), ("all_to_all_ms", ctypes.c_float), ("h_msm_ms", ctypes.c_float),
                ("witness_msms_ms", ctypes.c_float), ("witness_wait_ms", ctypes.c_float), ("gather_ms", ctypes.c_float),
                ("assemble_ms", ctypes.c_float), ("total_ms", ctypes.c_float)]

    def as_dict(self):
        return {f: getattr(self, f) for f, _ in self._fields_}


lib.zk_comm_unique_id.argtypes = [_vp]
lib.zk_comm_init_rank.argtypes = [ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp)]
lib.zk_comm_init_all.argtypes = [_vp, ctypes.c_int, _vp]
lib.zk_comm_init_local.argtypes = [ctypes.c_int, ctypes.c_int, _vp]
lib.zk_comm_abort.argtypes = [_vp]
lib.zk_comm_destroy.argtypes = [_vp]
lib.zk_comm_destroy.restype = None
lib.zk_groth16_prove_split.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]
lib.zk_groth16_split_last_stats.argtypes = [ctypes.POINTER(SplitStats)]
lib.zk_groth16_prove_multi.argtypes = [_vp, _vp, _vp, ctypes.c_int, _vp, _vp, _vp, _vp, _vp, ctypes.c_double, _vp]


class Comm:
    """One rank's communicator for zk_groth16_prove_split (zk_comm)."""

    def __init__(self, handle, keep=None):
        self.h = handle
        self._keep = keep

    @staticmethod
    def unique_id():
        """128-byte NCCL id (rank 0 makes it; the others receive it out of band)."""
        buf = (ctypes.c_uint8 * 128)()
        check(lib.zk_comm_unique_id(ctypes.cast(buf, _vp)))
        return bytes(buf)

    @classmethod
    def init_rank(cls, device, uid, nranks, rank):
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
        h = _vp()
        check(lib.zk_comm_init_rank(device, ctypes.cast(buf, _vp), nranks, rank, ctypes.byref(h)))
        return cls(h)

    @classmethod
    def init_all(cls, devices):
        arr = (ctypes.c_int * len(devices))(*devices)
        hs = (_vp * len(devices))()
        check(lib.zk_comm_init_all(ctypes.cast(arr, _vp), len(devices), ctypes.cast(hs, _vp)))
        return [cls(_vp(h)) for h in hs]

    @classmethod
    def init_local(cls, device, nranks):
        """nranks ranks as host threads sharing one device (no NCCL)."""
        hs = (_vp * nranks)()
        check(lib.zk_comm_init_local(device, nranks, ctypes.cast(hs, _vp)))
        return [cls(_vp(h)) for h in hs]

    def abort(self):
        check(lib.zk_comm_abort(self.h))

    def __del__(self):
        if getattr(self, "h", None):
            lib.zk_comm_destroy(self.h)
            self.h = None


def prove_split(pk, r1cs, comm, witness, r, s):
    """This rank's part of a proof split over comm's ranks (zk_groth16_prove_split):
    (proof bytes, A, B, C, per-phase statistics)."""
    witness = np.ascontiguousarray(witness, dtype=np.uint64)
    rr, ss = fr_from_int(r), fr_from_int(s)
    proof = np.zeros(256, np.uint8)
    pts = np.zeros(32, np.uint64)
    check(lib.zk_groth16_prove_split(pk.h, r1cs.h, comm.h, _np_ptr(witness), _np_ptr(rr), _np_ptr(ss), _np_ptr(proof), _np_ptr(pts)))
    st = SplitStats()
    lib.zk_groth16_split_last_stats(ctypes.byref(st))
    return proof.tobytes(), pts[:8], pts[8:24], pts[24:32], st.as_dict()


def prove_multi(pks, r1css, comms, witness, r, s, timeout_s=600.0):
    """All ranks from this thread (zk_groth16_prove_multi): (proof bytes, A, B, C,
    list of per-rank statistics)."""
    n = len(comms)
    witness = np.ascontiguousarray(witness, dtype=np.uint64)
    rr, ss = fr_from_int(r), fr_from_int(s)
    proof = np.zeros(256, np.uint8)
    pts = np.zeros(32, np.uint64)
    pk_arr = (_vp * n)(*[p.h for p in pks])
    r1_arr = (_vp * n)(*[x.h for x in r1css])
    cm_arr = (_vp * n)(*[c.h for c in comms])
    stats = (SplitStats * n)()
    check(lib.zk_groth16_prove_multi(ctypes.cast(pk_arr, _vp), ctypes.cast(r1_arr, _vp), ctypes.cast(cm_arr, _vp), n,
                                     _np_ptr(witness), _np_ptr(rr), _np_ptr(ss), _np_ptr(proof), _np_ptr(pts), timeout_s,
                                     ctypes.cast(stats, _vp)))
    return proof.tobytes(), pts[:8], pts[8:24], pts[24:32], [x.as_dict() for x in stats]


# ------------------------------------------------------------------ verifier
lib.zk_bn254_pairing.argtypes = [_vp, _vp, _vp]
lib.zk_bn254_pairing_check.argtypes = [_vp, _vp, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
lib.zk_groth16_vk_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(_vp)]
lib.zk_groth16_vk_from_pk.argtypes = [_vp, ctypes.POINTER(_vp)]
lib.zk_groth16_vk_destroy.argtypes = [_vp]
lib.zk_groth16_vk_destroy.restype = None
lib.zk_groth16_vk_num_public.argtypes = [_vp]
lib.zk_groth16_verify.argtypes = [_vp, ctypes.c_int, _vp, ctypes.c_int, _vp, ctypes.POINTER(ctypes.c_int)]


def bn254_pairing(p, q):
    """e(P, Q): packed G1 (8 words) and G2 (16 words) Montgomery -> (12, 4) uint64 Fp12."""
    p = np.ascontiguousarray(p, np.uint64)
    q = np.ascontiguousarray(q, np.uint64)
    out = np.zeros((12, 4), np.uint64)
    check(lib.zk_bn254_pairing(_np_ptr(p), _np_ptr(q), _np_ptr(out)))
    return out


def pairing_check(ps, qs):
    """prod_i e(P_i, Q_i) == 1 ?"""
    ps = np.ascontiguousarray(ps, np.uint64).reshape(-1, 8)
    qs = np.ascontiguousarray(qs, np.uint64).reshape(-1, 16)
    ok = ctypes.c_int(-1)
    check(lib.zk_bn254_pairing_check(_np_ptr(ps), _np_ptr(qs), ps.shape[0], ctypes.byref(ok)))
    return ok.value == 1


class VerifyingKey:
    """Groth16 verification key on the host (zk_groth16_vk)."""

    def __init__(self, handle):
        self.h = handle

    @classmethod
    def load(cls, path):
        h = _vp()
        check(lib.zk_groth16_vk_load(path.encode(), ctypes.byref(h)))
        return cls(h)

    @classmethod
    def from_pk(cls, pk):
        h = _vp()
        check(lib.zk_groth16_vk_from_pk(pk.h, ctypes.byref(h)))
        return cls(h)

    @property
    def num_public(self):
        return lib.zk_groth16_vk_num_public(self.h)

    def verify(self, public_inputs, proof, device=0):
        """Groth16 verification of 256 proof bytes against (n, 4) Montgomery public
        inputs; the public-input MSM on `device` (-1: on the host)."""
        pub = np.ascontiguousarray(public_inputs, np.uint64).reshape(-1, 4)
        pb = np.frombuffer(bytes(proof), dtype=np.uint8).copy()
        ok = ctypes.c_int(-1)
        check(lib.zk_groth16_verify(self.h, device, _np_ptr(pub) if pub.shape[0] else None, pub.shape[0], _np_ptr(pb),
                                    ctypes.byref(ok)))
        return ok.value == 1

    def __del__(self):
        if getattr(self, "h", None):
            lib.zk_groth16_vk_destroy(self.h)
            self.h = None


def prove_last_stats():
    s = ProveStats()
    check(lib.zk_groth16_last_stats(ctypes.byref(s)))
    return {"matvec_ms": s.matvec_ms, "compute_h_ms": s.compute_h_ms, "msm_ms": list(s.msm_ms), "total_ms": s.total_ms}
