// ref_driver.cpp -- exposes the reference's own host arithmetic through a C ABI
// so that the oracle restatement (bn254_oracle.c) and the golden fixtures can be
// pinned to it.
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile into oracle/_ref/ against
// the reference's headers where they lie (src/field/fp.cuh, src/field/fp2.cuh,
// src/curve/g1.cuh, src/curve/g2.cuh), with the reference's own host shim
// (tests/host/shim/cuda_runtime.h) standing in for the CUDA runtime, and linked
// with the reference's src/ntt/ntt.cu (compiled by nvcc) for compute_omega.
// Nothing from the reference is copied into this repository.
//
// All values cross this ABI in the reference's host layout: Montgomery-form
// 4 x u64 limbs; a G1 point is (x[4], y[4]) + an int infinity flag.
#include "field/fp.cuh"
#include "field/fp2.cuh"
#include "curve/g1.cuh"
#include "curve/g2.cuh"
#include "ntt/ntt.cuh"

#include <cstring>
#include <vector>

using namespace bn254;

static Fp ld_fp(const uint64_t* p) { return Fp(p[0], p[1], p[2], p[3]); }
static Fr ld_fr(const uint64_t* p) { return Fr(p[0], p[1], p[2], p[3]); }
static void st(uint64_t* o, const uint64_t* v) { std::memcpy(o, v, 32); }

static G1Affine ld_g1(const uint64_t* p, int inf) {
    if (inf) return G1Affine();
    return G1Affine(ld_fp(p), ld_fp(p + 4));
}
static void st_g1(uint64_t* o, int* inf, const G1Affine& a) {
    st(o, a.x.val); st(o + 4, a.y.val); *inf = a.infinity ? 1 : 0;
}
static G2Affine ld_g2(const uint64_t* p, int inf) {
    if (inf) return G2Affine();
    return G2Affine(Fp2(ld_fp(p), ld_fp(p + 4)), Fp2(ld_fp(p + 8), ld_fp(p + 12)));
}
static void st_g2(uint64_t* o, int* inf, const G2Affine& a) {
    st(o, a.x.c0.val); st(o + 4, a.x.c1.val); st(o + 8, a.y.c0.val); st(o + 12, a.y.c1.val);
    *inf = a.infinity ? 1 : 0;
}

extern "C" {

void ref_fp_mul(uint64_t* o, const uint64_t* a, const uint64_t* b) { st(o, (ld_fp(a) * ld_fp(b)).val); }
void ref_fp_add(uint64_t* o, const uint64_t* a, const uint64_t* b) { st(o, (ld_fp(a) + ld_fp(b)).val); }
void ref_fp_sub(uint64_t* o, const uint64_t* a, const uint64_t* b) { st(o, (ld_fp(a) - ld_fp(b)).val); }
void ref_fp_inv(uint64_t* o, const uint64_t* a) { st(o, ld_fp(a).inv().val); }
void ref_fr_mul(uint64_t* o, const uint64_t* a, const uint64_t* b) { st(o, (ld_fr(a) * ld_fr(b)).val); }
void ref_fr_add(uint64_t* o, const uint64_t* a, const uint64_t* b) { st(o, (ld_fr(a) + ld_fr(b)).val); }
void ref_fr_sub(uint64_t* o, const uint64_t* a, const uint64_t* b) { st(o, (ld_fr(a) - ld_fr(b)).val); }
void ref_fr_from_u64(uint64_t* o, uint64_t v) { st(o, Fr::from_uint(v).val); }
void ref_fr_to_std(uint64_t* o, const uint64_t* a) { ld_fr(a).to_standard(o); }
void ref_fp_to_std(uint64_t* o, const uint64_t* a) { ld_fp(a).to_standard(o); }
void ref_fp_from_std(uint64_t* o, const uint64_t* s) { st(o, Fp::from_standard(s[0], s[1], s[2], s[3]).val); }
void ref_fp_one(uint64_t* o) { st(o, Fp::one().val); }
void ref_fr_one(uint64_t* o) { st(o, Fr::one().val); }

void ref_compute_omega(uint64_t* o, int log_n, int inverse) {
    Fr w = inverse ? compute_omega_inv(log_n) : compute_omega(log_n);
    st(o, w.val);
}

void ref_g1_generator(uint64_t* o, int* inf) { st_g1(o, inf, G1Affine::generator()); }
void ref_g2_generator(uint64_t* o, int* inf) { st_g2(o, inf, G2Affine::generator()); }

// k * P (g1.cuh:204-246), returned affine
void ref_g1_scalar_mul(uint64_t* o, int* oinf, const uint64_t* p, int pinf, const uint64_t* k) {
    G1Jacobian j = G1Jacobian::from_affine(ld_g1(p, pinf)).scalar_mul(ld_fr(k));
    st_g1(o, oinf, j.to_affine());
}
// P + Q via Jacobian addition, P + Q via mixed addition, 2P via dbl
void ref_g1_add(uint64_t* o, int* oinf, const uint64_t* p, int pinf, const uint64_t* q, int qinf) {
    G1Jacobian j = G1Jacobian::from_affine(ld_g1(p, pinf)) + G1Jacobian::from_affine(ld_g1(q, qinf));
    st_g1(o, oinf, j.to_affine());
}
void ref_g1_madd(uint64_t* o, int* oinf, const uint64_t* p, int pinf, const uint64_t* q, int qinf) {
    G1Jacobian j = G1Jacobian::from_affine(ld_g1(p, pinf)).add_affine(ld_g1(q, qinf));
    st_g1(o, oinf, j.to_affine());
}
void ref_g1_dbl(uint64_t* o, int* oinf, const uint64_t* p, int pinf) {
    st_g1(o, oinf, G1Jacobian::from_affine(ld_g1(p, pinf)).dbl().to_affine());
}

void ref_g2_scalar_mul(uint64_t* o, int* oinf, const uint64_t* p, int pinf, const uint64_t* k) {
    G2Jacobian j = G2Jacobian::from_affine(ld_g2(p, pinf)).scalar_mul(ld_fr(k));
    st_g2(o, oinf, j.to_affine());
}
void ref_g2_add(uint64_t* o, int* oinf, const uint64_t* p, int pinf, const uint64_t* q, int qinf) {
    G2Jacobian j = G2Jacobian::from_affine(ld_g2(p, pinf)) + G2Jacobian::from_affine(ld_g2(q, qinf));
    st_g2(o, oinf, j.to_affine());
}
int ref_g2_on_curve(const uint64_t* p) { return ld_g2(p, 0).is_on_curve() ? 1 : 0; }
int ref_g1_on_curve(const uint64_t* p) { return ld_g1(p, 0).is_on_curve() ? 1 : 0; }

// The reference's small-n MSM path (src/msm/msm.cu:330-339), which is also its
// test oracle cpu_msm (tests/test_msm.cu:20-28).  points: n x (x[4], y[4]),
// an all-zero record is the identity.
void ref_msm_g1_naive(uint64_t* o, int* oinf, const uint64_t* pts, const uint64_t* sc, int n) {
    G1Jacobian acc = G1Jacobian::identity();
    for (int i = 0; i < n; i++) {
        const uint64_t* p = pts + 8 * i;
        int inf = 1;
        for (int k = 0; k < 8; k++) if (p[k]) inf = 0;
        acc = acc + G1Jacobian::from_affine(ld_g1(p, inf)).scalar_mul(ld_fr(sc + 4 * i));
    }
    st_g1(o, oinf, acc.to_affine());
}
void ref_msm_g2_naive(uint64_t* o, int* oinf, const uint64_t* pts, const uint64_t* sc, int n) {
    G2Jacobian acc = G2Jacobian::identity();
    for (int i = 0; i < n; i++) {
        const uint64_t* p = pts + 16 * i;
        int inf = 1;
        for (int k = 0; k < 16; k++) if (p[k]) inf = 0;
        acc = acc + G2Jacobian::from_affine(ld_g2(p, inf)).scalar_mul(ld_fr(sc + 4 * i));
    }
    st_g2(o, oinf, acc.to_affine());
}

// The reference's NTT test oracle: O(n^2) DFT with compute_omega
// (tests/test_ntt.cu:19-37), INTT scaled by (2^-1)^log_n as ntt.cu:437-459.
void ref_ntt_naive(uint64_t* out, const uint64_t* in, int log_n, int inverse) {
    int n = 1 << log_n;
    Fr omega = inverse ? compute_omega_inv(log_n) : compute_omega(log_n);
    std::vector<Fr> res(n);
    Fr omega_i = Fr::from_uint(1);
    for (int i = 0; i < n; i++) {
        Fr sum = Fr::zero();
        Fr wij = Fr::from_uint(1);
        for (int j = 0; j < n; j++) {
            sum = sum + ld_fr(in + 4 * j) * wij;
            wij = wij * omega_i;
        }
        res[i] = sum;
        omega_i = omega_i * omega;
    }
    if (inverse) {
        Fr two = Fr::from_uint(2);
        Fr half = two.inv();
        Fr scale = Fr::from_uint(1);
        for (int i = 0; i < log_n; i++) scale = scale * half;
        for (int i = 0; i < n; i++) res[i] = res[i] * scale;
    }
    for (int i = 0; i < n; i++) st(out + 4 * i, res[i].val);
}

}  // extern "C"

#include <thread>

// The reference's CPU MSM path run on `nthreads` host threads: each thread sums
// s_i * P_i over a contiguous slice with the reference's own scalar_mul and
// Jacobian addition (src/msm/msm.cu:330-339, src/curve/g1.cuh), and the slices
// are added at the end.  Used as the timed reference arm of bench.py.
extern "C" void ref_msm_g1_naive_mt(uint64_t* o, int* oinf, const uint64_t* pts, const uint64_t* sc, int n, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    std::vector<G1Jacobian> part(nthreads, G1Jacobian::identity());
    std::vector<std::thread> th;
    for (int t = 0; t < nthreads; t++) {
        th.emplace_back([&, t]() {
            int i0 = (int)((long long)n * t / nthreads), i1 = (int)((long long)n * (t + 1) / nthreads);
            G1Jacobian acc = G1Jacobian::identity();
            for (int i = i0; i < i1; i++) {
                const uint64_t* p = pts + 8 * i;
                int inf = 1;
                for (int k = 0; k < 8; k++) if (p[k]) inf = 0;
                acc = acc + G1Jacobian::from_affine(ld_g1(p, inf)).scalar_mul(ld_fr(sc + 4 * i));
            }
            part[t] = acc;
        });
    }
    G1Jacobian acc = G1Jacobian::identity();
    for (int t = 0; t < nthreads; t++) {
        th[t].join();
        acc = acc + part[t];
    }
    st_g1(o, oinf, acc.to_affine());
}

namespace bn254 {
void ntt_gpu(Fr* d_out, const Fr* d_in, int log_n, bool inverse);  // src/ntt/ntt.cuh:49 (ntt_ref.o)
}

// The reference's Pippenger MSM (src/msm/msm.cu:320-442) run on the host cores
// with the reference's own arithmetic: MSMConfig::for_size windows
// (src/msm/msm.cuh:46-63), unsigned c-bit digits of the standard-form scalar
// (msm.cu:122-142), zero digits and infinity points skipped, each nonzero digit
// added into its Jacobian bucket with G1Jacobian::add_affine (msm.cu:150-152),
// the per-window running-sum reduce (msm.cu:284-307) and the host combine with
// c doublings per window (msm.cu:423-430).  The windows are split over
// `nthreads` threads; the result is the canonical affine point.  This is the
// CPU baseline of bench.py's reference arm: the reference's algorithm and
// arithmetic without its GPU (whose buckets accumulate under unbounded spin
// locks, msm.cu:63-72, and are not run here).
extern "C" void ref_msm_g1_pippenger_mt(uint64_t* o, int* oinf, const uint64_t* pts, const uint64_t* sc, int n, int nthreads) {
    const int c = n <= (1 << 10) ? 10 : n <= (1 << 14) ? 12 : n <= (1 << 18) ? 14 : n <= (1 << 22) ? 15 : 16;
    const int W = (253 + c) / c;
    const int nb = (1 << c) - 1;
    std::vector<uint64_t> std_sc((size_t)n * 4);
    for (int i = 0; i < n; i++) ld_fr(sc + 4 * i).to_standard(&std_sc[(size_t)4 * i]);
    std::vector<G1Affine> P((size_t)n);
    for (int i = 0; i < n; i++) {
        const uint64_t* p = pts + 8 * i;
        int inf = 1;
        for (int k = 0; k < 8; k++) if (p[k]) inf = 0;
        P[(size_t)i] = ld_g1(p, inf);
    }
    std::vector<G1Jacobian> win((size_t)W, G1Jacobian::identity());
    if (nthreads < 1) nthreads = 1;
    std::vector<std::thread> th;
    for (int t = 0; t < nthreads; t++) {
        th.emplace_back([&, t]() {
            std::vector<G1Jacobian> bucket((size_t)nb);
            const uint64_t mask = ((uint64_t)1 << c) - 1;
            for (int w = t; w < W; w += nthreads) {
                std::fill(bucket.begin(), bucket.end(), G1Jacobian::identity());
                const int off = w * c, limb = off / 64, sh = off % 64;
                for (int i = 0; i < n; i++) {
                    if (P[(size_t)i].is_infinity()) continue;
                    const uint64_t* s = &std_sc[(size_t)4 * i];
                    uint64_t bits;
                    if (limb >= 4) bits = 0;
                    else if (sh + c <= 64) bits = (s[limb] >> sh) & mask;
                    else if (limb + 1 < 4) bits = ((s[limb] >> sh) | (s[limb + 1] << (64 - sh))) & mask;
                    else bits = (s[limb] >> sh) & mask;
                    if (bits == 0) continue;
                    bucket[(size_t)bits - 1] = bucket[(size_t)bits - 1].add_affine(P[(size_t)i]);
                }
                G1Jacobian running = G1Jacobian::identity(), sum = G1Jacobian::identity();
                for (int b = nb - 1; b >= 0; b--) {
                    if (!bucket[(size_t)b].is_infinity()) running = running + bucket[(size_t)b];
                    sum = sum + running;
                }
                win[(size_t)w] = sum;
            }
        });
    }
    for (auto& x : th) x.join();
    G1Jacobian r = G1Jacobian::identity();
    for (int w = W - 1; w >= 0; w--) {
        for (int i = 0; i < c; i++) r = r.dbl();
        r = r + win[(size_t)w];
    }
    st_g1(o, oinf, r.to_affine());
}

// The reference's own GPU NTT entry point bn254::ntt_gpu (src/ntt/ntt.cu:354-465,
// compiled for sm_100a from its source): device pointers, synchronous.
extern "C" void ref_ntt_gpu(void* d_out, const void* d_in, int log_n, int inverse) {
    bn254::ntt_gpu((bn254::Fr*)d_out, (const bn254::Fr*)d_in, log_n, inverse != 0);
}

// The reference's pairing e(P, Q) (src/curve/pairing.cuh:226-230) on its own
// host arithmetic: 12 Montgomery Fp in the Fp12 layout (c0.c0.c0 ... c1.c2.c1).
#include "curve/pairing.cuh"
extern "C" void ref_pairing(uint64_t* out48, const uint64_t* p, int pinf, const uint64_t* q, int qinf) {
    Fp12 e = pairing(ld_g1(p, pinf), ld_g2(q, qinf));
    const Fp6* h[2] = {&e.c0, &e.c1};
    for (int a = 0; a < 2; a++) {
        const Fp2* c[3] = {&h[a]->c0, &h[a]->c1, &h[a]->c2};
        for (int b = 0; b < 3; b++) {
            st(out48 + 4 * (a * 6 + b * 2), c[b]->c0.val);
            st(out48 + 4 * (a * 6 + b * 2 + 1), c[b]->c1.val);
        }
    }
}

// The ceremony's random linear combination sum_i rho_i P_i (src/prover/
// ceremony.cuh:242-246), the reference's own loop of scalar multiplications.
#include "prover/ceremony.cuh"
extern "C" void ref_random_combination(uint64_t* o, int* oinf, const uint64_t* pts, const uint64_t* rho, int n) {
    std::vector<G1Affine> p((size_t)n);
    std::vector<Fr> r((size_t)n);
    for (int i = 0; i < n; i++) {
        int inf = 1;
        for (int k = 0; k < 8; k++) if (pts[8 * i + k]) inf = 0;
        p[(size_t)i] = ld_g1(pts + 8 * i, inf);
        r[(size_t)i] = ld_fr(rho + 4 * i);
    }
    st_g1(o, oinf, zkml::ceremony::random_combination(p, r));
}
