"""The reference's own Groth16 code (src/prover/groth16.cu, compiled from its
sources into oracle/_ref/libzkref_g16.so, with msm_g1 / msm_g2 / ntt_gpu
resolved from this library) against this library's device prover on the same
circuit under the reference's deterministic seeds:
  * the 256-byte proofs are identical,
  * the ZKMLPK3 files written by ProvingKey::save and by zk_groth16_pk_save are
    identical,
  * Groth16Verifier::verify (the reference's host pairing) accepts this
    library's proof and rejects a tampered one."""
import ctypes
import os

import numpy as np
import pytest

import groth16_oracle as G
import zkml_b200 as Z

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "libzkref_g16.so")


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(LIB):
        pytest.skip("reference Groth16 driver not built (needs the reference tree at build time)")
    lib = ctypes.CDLL(LIB)
    vp, sz, i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
    lib.ref_g16_setup_prove.argtypes = [i, i, i, vp, sz, vp, sz, vp, sz, vp, vp, ctypes.POINTER(i), ctypes.c_char_p]
    lib.ref_g16_verify.argtypes = [i, i, i, vp, sz, vp, sz, vp, sz, vp, vp, ctypes.POINTER(i)]
    return lib


def _args(c):
    mats = [np.ascontiguousarray(c[k]) for k in "ABC"]
    return mats, [c["num_constraints"], c["num_variables"], c["num_public"],
                  mats[0].ctypes.data, len(mats[0]), mats[1].ctypes.data, len(mats[1]), mats[2].ctypes.data, len(mats[2])]


def test_reference_prover_and_verifier_agree(ref, tmp_path):
    c = Z.synth_conv_circuit(1, 2, 4, 4, 24, 10, 0, 2, 21)
    mats, a = _args(c)
    w = np.ascontiguousarray(c["witness"])
    ref_proof = np.zeros(256, np.uint8)
    ok = ctypes.c_int(-1)
    ref_pk = str(tmp_path / "ref_pk.bin")
    assert ref.ref_g16_setup_prove(*a, w.ctypes.data, ref_proof.ctypes.data, ctypes.byref(ok), ref_pk.encode()) == 0
    assert ok.value == 1, "the reference verifier rejected the reference's own proof"

    r1 = Z.R1cs(c)
    pk = Z.ProvingKey.setup(r1, G.toxic_deterministic())
    r, s = G.blinding_deterministic()
    proof, A, B, C = pk.prove(r1, w, r, s)
    assert proof == ref_proof.tobytes(), "proof bytes differ from the reference prover's"
    our_pk = str(tmp_path / "our_pk.bin")
    pk.save(our_pk)
    assert open(our_pk, "rb").read() == open(ref_pk, "rb").read(), "ZKMLPK3 bytes differ"

    pub = np.ascontiguousarray(w[1:1 + c["num_public"]])
    pb = np.frombuffer(proof, dtype=np.uint8).copy()
    assert ref.ref_g16_verify(*a, pub.ctypes.data, pb.ctypes.data, ctypes.byref(ok)) == 0
    assert ok.value == 1, "the reference verifier rejected this library's proof"
    pb[200] ^= 1
    assert ref.ref_g16_verify(*a, pub.ctypes.data, pb.ctypes.data, ctypes.byref(ok)) == 0
    assert ok.value == 0, "the reference verifier accepted a tampered proof"
