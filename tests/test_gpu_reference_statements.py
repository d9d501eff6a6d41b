"""Groth16 proofs of the reference's own statement-v2 circuits on the B200,
byte-for-byte against the reference's Groth16Prover::prove.

Circuits (built by the reference's build_statement_v2 through
oracle/ref_statements.py):
  * config 1: the quantised MLP 64 -> 32 (RELU_EXACT, 24 bits, shift 6) -> 10,
    int8 weights, inputs 0..16, batch 4, context-bound (7,762 constraints,
    domain 2^13);
  * the reference host test's tiny CNN, variant A (8,082 constraints);
  * config 4: its variant B, a Poseidon-committed private model with committed
    private inputs, private outputs and in-circuit routing (62,692
    constraints, domain 2^16).

For each: the proving and verification keys come from this library's device
setup under the reference's deterministic toxic waste (its ZKMLPK3 bytes equal
ProvingKey::save's, tests/test_gpu_reference_groth16.py); this library's proof
under the deterministic blinding must equal, byte for byte,
  * the reference's Groth16Prover::prove with msm_g1 / msm_g2 / ntt_gpu
    computed on the CPU by the oracle (no kernel of this library involved), and
  * the same reference prover linked against this library (the drop-in a
    zkml-prove user gets),
each loading the key files with ProvingKey::load_streaming and load_vk; the
reference's Groth16Verifier::verify accepts the proof and rejects it tampered."""
import os

import numpy as np
import pytest

import groth16_oracle as G
import ref_statements as RS
import zkml_b200 as Z

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def libs():
    for p in (RS.STMT_LIB, RS.G16_LIB, RS.G16_CPU_LIB):
        if not os.path.exists(p):
            pytest.skip(f"{os.path.basename(p)} not built (needs the reference tree at build time)")
    return RS.g16(RS.G16_CPU_LIB), RS.g16(RS.G16_LIB)


CASES = {
    "config1_mlp_b4": (lambda: RS.mlp_statement(), 7762, 7764, 298, 13),
    "tiny_cnn_A": (lambda: RS.tiny_cnn_statement("A"), 8082, 7868, 82, 13),
    "config4_tiny_cnn_B": (lambda: RS.tiny_cnn_statement("B"), 62692, 62779, 8, 16),
}


@pytest.mark.parametrize("name", list(CASES))
def test_statement_proof_equals_reference(libs, name, tmp_path):
    ref_cpu, ref_drop_in = libs
    build, nc, m, pub, log_n = CASES[name]
    c = build()
    assert (c["num_constraints"], c["num_variables"], c["num_public"]) == (nc, m, pub)
    r1 = Z.R1cs(c)
    assert r1.log_n == log_n
    pk = Z.ProvingKey.setup(r1, G.toxic_deterministic())
    pk_path, vk_path = str(tmp_path / "pk.bin"), str(tmp_path / "vk.bin")
    pk.save(pk_path)
    pk.save_vk(vk_path)
    r, s = G.blinding_deterministic()
    proof = pk.prove(r1, c["witness"], r, s)[0]
    assert pk.prove(r1, c["witness"], r, s)[0] == proof, "a second proof of the same inputs differs"

    ref_proof, ok, _ = RS.prove_with_keys(ref_cpu, pk_path, vk_path, c)
    assert ok, "the reference verifier rejected the reference's own proof"
    assert proof == ref_proof, "proof bytes differ from the reference prover's (CPU oracle MSM/NTT)"
    drop_proof, ok2, _ = RS.prove_with_keys(ref_drop_in, pk_path, vk_path, c)
    assert ok2 and drop_proof == proof, "the reference prover linked against this library gives another proof"

    assert RS.verify_with_vk(ref_cpu, vk_path, c, proof), "the reference verifier rejected this library's proof"
    bad = bytearray(proof)
    bad[200] ^= 1
    assert not RS.verify_with_vk(ref_cpu, vk_path, c, bytes(bad)), "the reference verifier accepted a tampered proof"

    # this library's verifier (public-input MSM on the GPU), from the key and from vk.bin
    pub = np.ascontiguousarray(c["witness"][1:1 + c["num_public"]])
    for vk in (Z.VerifyingKey.from_pk(pk), Z.VerifyingKey.load(vk_path)):
        assert vk.verify(pub, proof, device=0)
        assert not vk.verify(pub, bytes(bad), device=0)
        assert vk.verify(pub, proof, device=-1)


def test_statement_witness_refused_when_tampered(libs):
    """Flipping config 4's public route flag (the reference host test's
    negative check, tests/host/test_statement_v2.cpp:170-173) makes the
    witness unsatisfying: the device prover refuses it as the reference does."""
    c = RS.tiny_cnn_statement("B")
    r1 = Z.R1cs(c)
    pk = Z.ProvingKey.setup(r1, G.toxic_deterministic())
    w = c["witness"].copy()
    # public layout of variant B: tag, C_model, C_input x 2, then (flag, class) per sample
    flag = 1 + 4
    one = Z.fr_from_int(1)
    w[flag] = one if not np.array_equal(w[flag], one) else np.zeros(4, np.uint64)
    with pytest.raises(Z.ZkError) as e:
        pk.prove(r1, w, 1, 2)
    assert "does not satisfy" in str(e.value)
