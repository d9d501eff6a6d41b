// ref_groth16_driver.cu -- runs the reference's own Groth16 code
// (Groth16Prover::setup / prove, Groth16Proof::serialize / deserialize,
// ProvingKey::save, Groth16Verifier::verify from src/prover/groth16.cu, and
// the host pairing of src/curve/pairing.cuh) on a given R1CS and witness.
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile into oracle/_ref/ from
// the reference's sources where they lie, and linked against
// libzkml_b200.so, which supplies bn254::msm_g1 / msm_g2 / ntt_gpu /
// compute_omega in place of the reference's src/msm/msm.cu and src/ntt/ntt.cu
// -- exactly the drop-in the library is for.  Used on the GPU box to check
// that the library's own prover produces the reference's proof and proving-key
// bytes and that the reference's verifier accepts its proofs.
#include "prover/groth16.cuh"
#include "verifier/verifier.cuh"

#include <unistd.h>

#include <chrono>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

using namespace zkml;

static R1CS make_r1cs(int nc, int m, int pub, const void* a, size_t na, const void* b, size_t nb, const void* c, size_t nc3) {
    R1CS r;
    r.num_constraints = nc;
    r.num_variables = m;
    r.num_public_inputs = pub;
    r.num_private_inputs = m - 1 - pub;
    r.A.resize(na);
    r.B.resize(nb);
    r.C.resize(nc3);
    static_assert(sizeof(SparseEntry) == 40, "SparseEntry layout");
    std::memcpy(r.A.data(), a, na * sizeof(SparseEntry));
    std::memcpy(r.B.data(), b, nb * sizeof(SparseEntry));
    std::memcpy(r.C.data(), c, nc3 * sizeof(SparseEntry));
    return r;
}

extern "C" {

// Deterministic setup + prove with the reference's code.  Writes the 256-byte
// proof, the verifier's verdict on it, and (if pk_path) the ZKMLPK3 file.
int ref_g16_setup_prove(int nc, int m, int pub, const void* a, size_t na, const void* b, size_t nb, const void* c, size_t ncc,
                        const void* witness, uint8_t* proof_out, int* verified, const char* pk_path) {
    setenv("ZKML_DETERMINISTIC_SETUP", "1", 1);
    setenv("ZKML_DETERMINISTIC_PROVE", "1", 1);
    R1CS r = make_r1cs(nc, m, pub, a, na, b, nb, c, ncc);
    Witness w;
    w.values.resize(m);
    std::memcpy(w.values.data(), witness, (size_t)m * sizeof(bn254::Fr));
    w.num_public = pub;
    w.num_private = m - 1 - pub;
    ProvingKey pk;
    VerificationKey vk;
    Groth16Prover::setup(r, pk, vk);
    if (pk_path && !pk.save(pk_path)) return 2;
    Groth16Proof proof = Groth16Prover::prove(pk, r, w);
    if (!proof.valid) return 3;
    std::vector<uint8_t> bytes = proof.serialize();
    std::memcpy(proof_out, bytes.data(), 256);
    *verified = Groth16Verifier::verify(vk, proof, w.get_public()) ? 1 : 0;
    return 0;
}

// The reference's verifier on externally produced proof bytes, with the
// verification key of the deterministic setup of the same circuit.  The proof
// goes through the CLI's reader, load_proof (src/verifier/verifier.cu:47-101):
// Groth16Proof::deserialize (src/prover/groth16.cu:1076-1094) builds each point
// as G1Affine(read_fp(ptr), read_fp(ptr)), whose argument order is unspecified
// in C++ (GCC reads y first), so it does not round-trip serialize().
int ref_g16_verify(int nc, int m, int pub, const void* a, size_t na, const void* b, size_t nb, const void* c, size_t ncc,
                   const void* public_inputs, const uint8_t* proof_bytes, int* verified) {
    setenv("ZKML_DETERMINISTIC_SETUP", "1", 1);
    R1CS r = make_r1cs(nc, m, pub, a, na, b, nb, c, ncc);
    ProvingKey pk;
    VerificationKey vk;
    Groth16Prover::setup(r, pk, vk);
    char path[] = "/tmp/zkref_proof_XXXXXX";
    int fd = mkstemp(path);
    if (fd < 0) return 4;
    bool wrote = write(fd, proof_bytes, 256) == 256;
    close(fd);
    if (!wrote) { unlink(path); return 4; }
    Groth16Proof proof = load_proof(path);
    unlink(path);
    std::vector<bn254::Fr> pubs((size_t)pub);
    std::memcpy(pubs.data(), public_inputs, (size_t)pub * sizeof(bn254::Fr));
    *verified = Groth16Verifier::verify(vk, proof, pubs) ? 1 : 0;
    return 0;
}

// The reference's Groth16Prover::prove from key files: a ZKMLPK3 proving key
// read by ProvingKey::load_streaming (src/prover/groth16.cu:1190-1314) and a
// vk.bin read by load_vk (src/verifier/verifier.cu:103-148), both written by
// the library under test (its setup is byte-identical to the reference's, and
// the reference's own host setup would take minutes to hours at the larger
// configurations).  Deterministic blinding (ZKML_DETERMINISTIC_PROVE=1).
// Writes the 256-byte proof, the reference verifier's verdict on it, and the
// wall time of prove() in milliseconds.
int ref_g16_prove_keys(const char* pk_path, const char* vk_path, int nc, int m, int pub, const void* a, size_t na, const void* b,
                       size_t nb, const void* c, size_t ncc, const void* witness, uint8_t* proof_out, int* verified,
                       double* prove_ms) {
    setenv("ZKML_DETERMINISTIC_PROVE", "1", 1);
    R1CS r = make_r1cs(nc, m, pub, a, na, b, nb, c, ncc);
    Witness w;
    w.values.resize(m);
    std::memcpy(w.values.data(), witness, (size_t)m * sizeof(bn254::Fr));
    w.num_public = pub;
    w.num_private = m - 1 - pub;
    ProvingKey pk;
    if (!pk.load_streaming(pk_path)) return 2;
    VerificationKey vk = load_vk(vk_path);
    if ((int)vk.ic.size() != pub + 1) return 5;
    auto t0 = std::chrono::steady_clock::now();
    Groth16Proof proof = Groth16Prover::prove(pk, r, w);
    auto t1 = std::chrono::steady_clock::now();
    if (prove_ms) *prove_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
    if (!proof.valid) return 3;
    std::vector<uint8_t> bytes = proof.serialize();
    std::memcpy(proof_out, bytes.data(), 256);
    *verified = Groth16Verifier::verify(vk, proof, w.get_public()) ? 1 : 0;
    return 0;
}

// The reference verifier on externally produced proof bytes with a vk.bin
// (load_vk) instead of a setup: reads the proof through load_proof as the CLI does.
int ref_g16_verify_vk(const char* vk_path, int pub, const void* public_inputs, const uint8_t* proof_bytes, int* verified) {
    VerificationKey vk = load_vk(vk_path);
    if ((int)vk.ic.size() != pub + 1) return 5;
    char path[] = "/tmp/zkref_proof_XXXXXX";
    int fd = mkstemp(path);
    if (fd < 0) return 4;
    bool wrote = write(fd, proof_bytes, 256) == 256;
    close(fd);
    if (!wrote) { unlink(path); return 4; }
    Groth16Proof proof = load_proof(path);
    unlink(path);
    std::vector<bn254::Fr> pubs((size_t)pub);
    std::memcpy(pubs.data(), public_inputs, (size_t)pub * sizeof(bn254::Fr));
    *verified = Groth16Verifier::verify(vk, proof, pubs) ? 1 : 0;
    return 0;
}

}  // extern "C"
