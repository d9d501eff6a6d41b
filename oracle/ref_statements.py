"""Circuits built by the reference's own statement-v2 builder
(build_statement_v2, src/prover/statement_v2.cuh:82-257), through
oracle/_ref/libzkref_stmt.so (test infrastructure, built by oracle/Makefile
from the reference tree), and the reference's Groth16 prover/verifier entry
points of oracle/ref_groth16_driver.cu.  Test and measurement infrastructure:
used by the tests and by bench.py's reference arm only.

Circuits come back in the layout of zkml_b200.synth_*: SparseEntry arrays A, B,
C, the witness (num_variables x 4 Montgomery limbs) and the counts."""
import ctypes
import os

import numpy as np

import zkml_b200 as Z

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
STMT_LIB = os.path.join(REF_DIR, "libzkref_stmt.so")
G16_LIB = os.path.join(REF_DIR, "libzkref_g16.so")          # reference Groth16 + this library's msm/ntt
G16_CPU_LIB = os.path.join(REF_DIR, "libzkref_g16_cpu.so")  # reference Groth16 + the CPU oracle's msm/ntt

_vp, _sz, _i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int


class _RefCircuit(ctypes.Structure):
    _fields_ = [("num_constraints", _i), ("num_variables", _i), ("num_public", _i),
                ("nnz", _sz * 3), ("entries", _vp * 3), ("witness", _vp)]


_stmt = None


def available():
    return os.path.exists(STMT_LIB)


def _lib():
    global _stmt
    if _stmt is None:
        _stmt = ctypes.CDLL(STMT_LIB)
        _stmt.ref_stmt_mlp.argtypes = [_i] * 7 + [ctypes.c_uint64] + [_vp] * 6
        _stmt.ref_stmt_tiny_cnn.argtypes = [_i, _vp]
        _stmt.ref_circuit_free.argtypes = [_vp]
        _stmt.ref_circuit_free.restype = None
    return _stmt


def _copy(c):
    lib = _lib()
    try:
        mats = []
        for k in range(3):
            nbytes = 40 * c.nnz[k]
            raw = np.ctypeslib.as_array((ctypes.c_uint8 * max(nbytes, 1)).from_address(c.entries[k]))[:nbytes]
            mats.append(raw.copy().view(Z.ENTRY_DTYPE))
        m = c.num_variables
        w = np.ctypeslib.as_array((ctypes.c_uint64 * (4 * m)).from_address(c.witness)).copy().reshape(m, 4)
        return {"A": mats[0], "B": mats[1], "C": mats[2], "witness": w, "num_constraints": c.num_constraints,
                "num_variables": m, "num_public": c.num_public}
    finally:
        lib.ref_circuit_free(ctypes.byref(c))


def mlp_model(n_in=64, n_hidden=32, n_out=10, batch=4, seed=1):
    """int8 weights and biases uniform in [-127, 127], inputs uniform in [0, 16]."""
    rng = np.random.default_rng(seed)
    return {"w1": rng.integers(-127, 128, (n_hidden, n_in)).astype(np.int32),
            "b1": rng.integers(-127, 128, n_hidden).astype(np.int32),
            "w2": rng.integers(-127, 128, (n_out, n_hidden)).astype(np.int32),
            "b2": rng.integers(-127, 128, n_out).astype(np.int32),
            "x": rng.integers(0, 17, (batch, n_in)).astype(np.int32)}


def mlp_statement(batch=4, n_in=64, n_hidden=32, n_out=10, bits=24, shift=6, context=True, seed=1, tag=0xC0FFEE):
    """The quantised MLP statement (LINEAR + RELU_EXACT, LINEAR; public inputs
    and outputs, model tag, context-bound) built by the reference."""
    md = mlp_model(n_in, n_hidden, n_out, batch, seed)
    c = _RefCircuit()
    p = [np.ascontiguousarray(md[k]).ctypes.data for k in ("w1", "b1", "w2", "b2", "x")]
    rc = _lib().ref_stmt_mlp(batch, n_in, n_hidden, n_out, bits, shift, int(context), tag, *p, ctypes.byref(c))
    if rc != 0:
        raise RuntimeError(f"reference statement builder failed ({rc})")
    return _copy(c)


def tiny_cnn_statement(variant):
    """The reference host test's tiny-CNN statement: variant 'A' (public,
    context-bound) or 'B' (private model and inputs, routing)."""
    c = _RefCircuit()
    rc = _lib().ref_stmt_tiny_cnn({"A": 0, "B": 1}[variant], ctypes.byref(c))
    if rc != 0:
        raise RuntimeError(f"reference statement builder failed ({rc})")
    return _copy(c)


def g16(path):
    lib = ctypes.CDLL(path)
    lib.ref_g16_setup_prove.argtypes = [_i, _i, _i, _vp, _sz, _vp, _sz, _vp, _sz, _vp, _vp, ctypes.POINTER(_i), ctypes.c_char_p]
    lib.ref_g16_verify.argtypes = [_i, _i, _i, _vp, _sz, _vp, _sz, _vp, _sz, _vp, _vp, ctypes.POINTER(_i)]
    lib.ref_g16_prove_keys.argtypes = [ctypes.c_char_p, ctypes.c_char_p, _i, _i, _i, _vp, _sz, _vp, _sz, _vp, _sz, _vp, _vp,
                                       ctypes.POINTER(_i), ctypes.POINTER(ctypes.c_double)]
    lib.ref_g16_verify_vk.argtypes = [ctypes.c_char_p, _i, _vp, _vp, ctypes.POINTER(_i)]
    return lib


def circuit_args(c):
    """(kept-alive arrays, the nc, m, pub, A, nA, B, nB, C, nC argument list)."""
    mats = [np.ascontiguousarray(c[k]) for k in "ABC"]
    return mats, [c["num_constraints"], c["num_variables"], c["num_public"],
                  mats[0].ctypes.data, len(mats[0]), mats[1].ctypes.data, len(mats[1]), mats[2].ctypes.data, len(mats[2])]


def prove_with_keys(lib, pk_path, vk_path, c):
    """The reference's Groth16Prover::prove from key files (deterministic
    blinding): (proof bytes, verified by Groth16Verifier::verify, prove ms)."""
    mats, a = circuit_args(c)
    w = np.ascontiguousarray(c["witness"])
    out = np.zeros(256, np.uint8)
    ok = ctypes.c_int(-1)
    ms = ctypes.c_double(0)
    rc = lib.ref_g16_prove_keys(pk_path.encode(), vk_path.encode(), *a, w.ctypes.data, out.ctypes.data, ctypes.byref(ok),
                                ctypes.byref(ms))
    if rc != 0:
        raise RuntimeError(f"reference prove from key files failed ({rc})")
    return out.tobytes(), ok.value == 1, ms.value


def verify_with_vk(lib, vk_path, c, proof):
    pub = np.ascontiguousarray(c["witness"][1:1 + c["num_public"]])
    pb = np.frombuffer(proof, dtype=np.uint8).copy()
    ok = ctypes.c_int(-1)
    rc = lib.ref_g16_verify_vk(vk_path.encode(), c["num_public"], pub.ctypes.data, pb.ctypes.data, ctypes.byref(ok))
    if rc != 0:
        raise RuntimeError(f"reference verify failed ({rc})")
    return ok.value == 1
