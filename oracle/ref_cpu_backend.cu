// ref_cpu_backend.cu -- bn254::msm_g1 / msm_g2 / ntt_gpu / compute_omega for
// the reference's own Groth16 code, computed on the CPU by the oracle (the
// plain-C restatement of the reference's Pippenger MSM and radix-2 NTT,
// bn254_oracle.c).
//
// TEST INFRASTRUCTURE ONLY.  Linked by oracle/Makefile with the reference's
// src/prover/groth16.cu and src/verifier/verifier.cu (compiled from its tree)
// into oracle/_ref/libzkref_g16_cpu.so, so that the reference's
// Groth16Prover::prove runs with no kernel of the library under test: its
// proofs are then an independent check of that library's device prover.  The
// reference's own MSM kernels are not used (their buckets accumulate under
// unbounded atomicCAS spin locks, src/msm/msm.cu:63-72).
//
// Same interface as src/msm/msm.cuh:67-68 and src/ntt/ntt.cuh:49-54: the MSMs
// take host arrays, ntt_gpu device pointers (copied to the host and back).
#include "curve/g1.cuh"
#include "curve/g2.cuh"
#include "field/fp.cuh"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "bn254_oracle.h"

namespace {
int threads() {
    const unsigned t = std::thread::hardware_concurrency();
    return t ? (int)t : 1;
}
void fail(const char* what, cudaError_t e) {
    fprintf(stderr, "ref_cpu_backend: %s: %s\n", what, cudaGetErrorString(e));
    exit(EXIT_FAILURE);  // the reference's CUDA_CHECK convention (src/common.cuh:11-19)
}
}  // namespace

namespace bn254 {

Fr compute_omega(int log_n) {
    orc_fe w;
    orc_compute_omega(&w, log_n, 0);
    return Fr(w.v[0], w.v[1], w.v[2], w.v[3]);
}

Fr compute_omega_inv(int log_n) {
    orc_fe w;
    orc_compute_omega(&w, log_n, 1);
    return Fr(w.v[0], w.v[1], w.v[2], w.v[3]);
}

G1Jacobian msm_g1(const G1Affine* h_points, const Fr* h_scalars, int n) {
    if (n <= 0) return G1Jacobian::identity();
    std::vector<uint64_t> pts((size_t)n * 8, 0);  // packed (x, y); all-zero = infinity
    for (int i = 0; i < n; i++)
        if (!h_points[i].infinity) {
            std::memcpy(&pts[(size_t)i * 8], h_points[i].x.val, 32);
            std::memcpy(&pts[(size_t)i * 8 + 4], h_points[i].y.val, 32);
        }
    orc_g1a r;
    orc_msm_g1(&r, pts.data(), reinterpret_cast<const uint64_t*>(h_scalars), (size_t)n, threads());
    if (r.inf) return G1Jacobian::identity();
    return G1Jacobian(Fp(r.x.v[0], r.x.v[1], r.x.v[2], r.x.v[3]), Fp(r.y.v[0], r.y.v[1], r.y.v[2], r.y.v[3]), Fp::one());
}

G2Jacobian msm_g2(const G2Affine* h_points, const Fr* h_scalars, int n) {
    if (n <= 0) return G2Jacobian::identity();
    std::vector<uint64_t> pts((size_t)n * 16, 0);
    for (int i = 0; i < n; i++)
        if (!h_points[i].infinity) {
            std::memcpy(&pts[(size_t)i * 16], h_points[i].x.c0.val, 32);
            std::memcpy(&pts[(size_t)i * 16 + 4], h_points[i].x.c1.val, 32);
            std::memcpy(&pts[(size_t)i * 16 + 8], h_points[i].y.c0.val, 32);
            std::memcpy(&pts[(size_t)i * 16 + 12], h_points[i].y.c1.val, 32);
        }
    orc_g2a r;
    orc_msm_g2(&r, pts.data(), reinterpret_cast<const uint64_t*>(h_scalars), (size_t)n, threads());
    if (r.inf) return G2Jacobian::identity();
    auto fp = [](const orc_fe& f) { return Fp(f.v[0], f.v[1], f.v[2], f.v[3]); };
    return G2Jacobian(Fp2(fp(r.x.c0), fp(r.x.c1)), Fp2(fp(r.y.c0), fp(r.y.c1)), Fp2::one());
}

void ntt_gpu(Fr* d_out, const Fr* d_in, int log_n, bool inverse) {
    if (log_n < 0 || log_n > 24) {  // gpu_config::NTT_MAX_LOG (src/common.cuh:78); ntt.cu:357-361
        fprintf(stderr, "NTT size 2^%d exceeds limit 2^24\n", log_n);
        return;
    }
    const size_t n = (size_t)1 << log_n;
    std::vector<uint64_t> in(n * 4), out(n * 4);
    cudaError_t e = cudaMemcpy(in.data(), d_in, n * 32, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) fail("copy in", e);
    orc_ntt_mt(out.data(), in.data(), log_n, inverse ? 1 : 0, threads());
    e = cudaMemcpy(d_out, out.data(), n * 32, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) fail("copy out", e);
}

void ntt_gpu_inplace(Fr* d_data, int log_n, bool inverse) { ntt_gpu(d_data, d_data, log_n, inverse); }

}  // namespace bn254
