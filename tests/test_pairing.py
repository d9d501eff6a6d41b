"""The BN254 optimal ate pairing and the Groth16 verifier of this library
(host code; zk_bn254_pairing, zk_bn254_pairing_check, zk_groth16_verify with
the public-input sum on the host, device = -1), on the CPU:
  * pairing values equal, bit for bit, the reference's bn254::pairing
    (src/curve/pairing.cuh:226-230, its host arithmetic compiled into
    oracle/_ref/libzkref.so);
  * bilinearity and non-degeneracy through the pairing-product check;
  * the verifier accepts the reference's own Groth16 proofs made on a T4
    (results/gpu_validation_2026/artifacts: vk.bin, proofs, public inputs,
    read in place) and rejects tampered ones."""
import glob
import os

import numpy as np
import pytest

import pyoracle as O
import zkml_b200 as Z

P_MOD = 21888242871839275222246405745257275088696311157297823662689037894645226208583
ART = os.path.join(O.reference_tree(), "results", "gpu_validation_2026", "artifacts")


def neg_g1(p):
    """-P for a packed Montgomery G1 point (p - y is the Montgomery form of -y)."""
    q = np.array(p, copy=True)
    v = (P_MOD - O.to_int(p[4:8])) % P_MOD
    q[4:8] = [(v >> (64 * i)) & (2**64 - 1) for i in range(4)]
    return q


@pytest.fixture(scope="module")
def pts():
    rng = O.Rng(77)
    k = rng.fr_vector(6)
    return k, O.g1_fixed_base(k[:3]), O.g2_fixed_base(k[3:])


@pytest.mark.skipif(not O.ref_available(), reason="reference arithmetic not built")
def test_pairing_equals_reference(pts):
    import ctypes
    _, P, Q = pts
    ref = O.ref()
    for i in range(3):
        out = np.zeros(48, np.uint64)
        ref.ref_pairing(O._p(out), O._p(P[i]), 0, O._p(Q[i]), 0)
        assert np.array_equal(Z.bn254_pairing(P[i], Q[i]).reshape(-1), out), i
    # e(O, Q) = e(P, O) = 1
    one = Z.bn254_pairing(np.zeros(8, np.uint64), Q[0])
    assert np.array_equal(one[0], O.fp_from_int(1)) and not one[1:].any()
    assert np.array_equal(Z.bn254_pairing(P[0], np.zeros(16, np.uint64)), one)
    _ = ctypes


def test_bilinearity(pts):
    k, P, Q = pts
    a = k[5]
    aP = O.g1_fixed_base(O.fr_mul(k[0], a)[None, :])[0]
    aQ = O.g2_fixed_base(O.fr_mul(k[3], a)[None, :])[0]
    # e(aP, Q) e(-P, aQ) = 1, and not with another Q
    assert Z.pairing_check(np.stack([aP, neg_g1(P[0])]), np.stack([Q[0], aQ]))
    assert not Z.pairing_check(np.stack([aP, neg_g1(P[0])]), np.stack([Q[0], Q[1]]))
    # e(P, Q) e(-P, Q) = 1; e(P, Q) != 1
    assert Z.pairing_check(np.stack([P[1], neg_g1(P[1])]), np.stack([Q[2], Q[2]]))
    assert not Z.pairing_check(P[1][None, :], Q[2][None, :])
    assert Z.pairing_check(np.zeros((0, 8), np.uint64), np.zeros((0, 16), np.uint64))


def _artifacts():
    out = []
    for case in ("p16", "p48", "p96", "p160"):
        d = os.path.join(ART, case)
        for pf in sorted(glob.glob(os.path.join(d, "*.proof.bin")))[:2]:
            out.append((case, pf))
    return out


@pytest.mark.skipif(not os.path.isdir(ART), reason="reference artefacts not present")
@pytest.mark.parametrize("case,proof_path", _artifacts() or [("none", "")])
def test_verifies_reference_t4_proofs(case, proof_path):
    vk = Z.VerifyingKey.load(os.path.join(ART, case, "vk.bin"))
    raw = open(proof_path.replace(".proof.bin", ".public.bin"), "rb").read()
    n = int.from_bytes(raw[:4], "little")
    pub = O.fr_from_std_vector(np.frombuffer(raw[4:4 + 32 * n], dtype=np.uint64).reshape(n, 4))
    proof = open(proof_path, "rb").read()
    assert vk.num_public == n
    assert vk.verify(pub, proof, device=-1)
    bad = bytearray(proof)
    bad[100] ^= 1
    assert not vk.verify(pub, bytes(bad), device=-1)
    wrong = pub.copy()
    wrong[0] = O.fr_from_int(O.to_int(wrong[0]) * 7)  # another field element
    assert not vk.verify(wrong, proof, device=-1)
    assert not vk.verify(pub[:-1], proof, device=-1)   # wrong public-input count
