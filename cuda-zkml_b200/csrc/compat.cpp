// compat.cpp -- the reference's C++ entry points, re-exported over the C ABI.
//
// gdtsitlauri/cuda-zkml calls its hot path through these functions
// (src/msm/msm.cuh:67-68, src/ntt/ntt.cuh:49-54); its prover
// (src/prover/groth16.cu:111, :316, :399, :436, :776, :792, :810, :817, :827)
// and tests link them from the static libraries zkml_msm / zkml_ntt
// (CMakeLists.txt:74-90).  This file defines the same symbols so that code links
// against libzkml_b200 unchanged.  The structs below repeat only the data layout
// of the reference's types (field limbs, coordinates, the infinity flag), which
// is what the symbols and the by-value returns depend on; the mangled names
// carry only namespace and type names.
//
// Error behaviour follows the reference: a CUDA failure prints and exits
// (CUDA_CHECK, src/common.cuh:11-19); ntt_gpu with log_n > 24 prints an error
// and returns with the output untouched (src/ntt/ntt.cu:357-361).
#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include "../../include/zkml_b200.h"

namespace bn254 {

struct Fp {
    uint64_t val[4];
};
struct Fr {
    uint64_t val[4];
};
struct Fp2 {
    Fp c0, c1;
};
struct G1Affine {
    Fp x, y;
    bool infinity;
};
struct G1Jacobian {
    Fp x, y, z;
};
struct G2Affine {
    Fp2 x, y;
    bool infinity;
};
struct G2Jacobian {
    Fp2 x, y, z;
};

static_assert(sizeof(G1Affine) == 72, "G1Affine layout");
static_assert(sizeof(G2Affine) == 136, "G2Affine layout");
static_assert(sizeof(G1Jacobian) == 96, "G1Jacobian layout");
static_assert(sizeof(G2Jacobian) == 192, "G2Jacobian layout");

static void die_on(int status, const char* what) {
    if (status == ZK_OK) return;
    fprintf(stderr, "CUDA error in %s: %s\n", what, zk_last_error());
    exit(EXIT_FAILURE);
}

G1Jacobian msm_g1(const G1Affine* h_points, const Fr* h_scalars, int n);
G2Jacobian msm_g2(const G2Affine* h_points, const Fr* h_scalars, int n);
void ntt_gpu(Fr* d_out, const Fr* d_in, int log_n, bool inverse);
void ntt_gpu_inplace(Fr* d_data, int log_n, bool inverse);
Fr compute_omega(int log_n);
Fr compute_omega_inv(int log_n);

G1Jacobian msm_g1(const G1Affine* h_points, const Fr* h_scalars, int n) {
    G1Jacobian r;
    die_on(zk_msm_g1(h_points, h_scalars, n, &r), "msm_g1");
    return r;
}

G2Jacobian msm_g2(const G2Affine* h_points, const Fr* h_scalars, int n) {
    G2Jacobian r;
    die_on(zk_msm_g2(h_points, h_scalars, n, &r), "msm_g2");
    return r;
}

void ntt_gpu(Fr* d_out, const Fr* d_in, int log_n, bool inverse) {
    if (log_n > ZK_REF_NTT_MAX_LOG) {
        fprintf(stderr, "[NTT] Error: log_n=%d exceeds max %d\n", log_n, ZK_REF_NTT_MAX_LOG);
        return;
    }
    die_on(zk_ntt(d_out, d_in, log_n, inverse ? 1 : 0), "ntt_gpu");
}

void ntt_gpu_inplace(Fr* d_data, int log_n, bool inverse) {
    if (log_n > ZK_REF_NTT_MAX_LOG) {
        fprintf(stderr, "[NTT] Error: log_n=%d exceeds max %d\n", log_n, ZK_REF_NTT_MAX_LOG);
        return;
    }
    die_on(zk_ntt_inplace(d_data, log_n, inverse ? 1 : 0), "ntt_gpu_inplace");
}

Fr compute_omega(int log_n) {
    Fr r = {{0, 0, 0, 0}};
    if (zk_compute_omega(log_n, 0, &r) != ZK_OK) die_on(ZK_ERR_INVALID, "compute_omega");
    return r;
}

Fr compute_omega_inv(int log_n) {
    Fr r = {{0, 0, 0, 0}};
    if (zk_compute_omega(log_n, 1, &r) != ZK_OK) die_on(ZK_ERR_INVALID, "compute_omega_inv");
    return r;
}

}  // namespace bn254
