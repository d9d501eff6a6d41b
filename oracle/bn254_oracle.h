/*
 * bn254_oracle.h -- CPU restatement of gdtsitlauri/cuda-zkml's Groth16 proving
 * hot path (BN254 field/curve arithmetic, Pippenger MSM, radix-2 NTT).
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may load
 * it.  The product library (cuda-zkml_b200/) never links, calls or falls back
 * to it.
 *
 * Parity pin: every function here is checked against the reference's own host
 * arithmetic (src/field/fp.cuh, src/curve/g1.cuh, src/curve/g2.cuh compiled
 * with g++ from the reference tree by oracle/Makefile into oracle/_ref/) through
 * the golden vectors in tests/golden/.
 *
 * Data layout (identical to the reference's host structs):
 *   field element  : 4 x uint64 little-endian limbs, Montgomery form (R = 2^256)
 *   G1 affine      : x[4], y[4]  (+ separate infinity flag)
 *   G1 Jacobian    : X[4], Y[4], Z[4]; identity = (0, one, 0)
 *   G2             : every Fp becomes Fp2 = (c0[4], c1[4])
 */
#ifndef BN254_ORACLE_H
#define BN254_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct { uint64_t v[4]; } orc_fe;           /* Fp or Fr, Montgomery */
typedef struct { orc_fe c0, c1; } orc_fe2;          /* Fp2 = Fp[u]/(u^2+1) */
typedef struct { orc_fe x, y; int inf; } orc_g1a;   /* G1 affine */
typedef struct { orc_fe x, y, z; } orc_g1j;         /* G1 Jacobian */
typedef struct { orc_fe2 x, y; int inf; } orc_g2a;  /* G2 affine */
typedef struct { orc_fe2 x, y, z; } orc_g2j;        /* G2 Jacobian */

/* ---- base field Fp (src/field/fp.cuh:30-314, montgomery.cuh:33-60) ---- */
void orc_fp_mul(orc_fe* r, const orc_fe* a, const orc_fe* b);
void orc_fp_add(orc_fe* r, const orc_fe* a, const orc_fe* b);
void orc_fp_sub(orc_fe* r, const orc_fe* a, const orc_fe* b);
void orc_fp_neg(orc_fe* r, const orc_fe* a);
void orc_fp_inv(orc_fe* r, const orc_fe* a);
void orc_fp_from_std(orc_fe* r, const uint64_t s[4]);
void orc_fp_to_std(uint64_t s[4], const orc_fe* a);
void orc_fp_one(orc_fe* r);

/* ---- scalar field Fr (src/field/fp.cuh:322-583) ---- */
void orc_fr_mul(orc_fe* r, const orc_fe* a, const orc_fe* b);
void orc_fr_add(orc_fe* r, const orc_fe* a, const orc_fe* b);
void orc_fr_sub(orc_fe* r, const orc_fe* a, const orc_fe* b);
void orc_fr_inv(orc_fe* r, const orc_fe* a);
void orc_fr_from_std(orc_fe* r, const uint64_t s[4]);
/* n standard-form values (4 limbs each, < r) to Montgomery form */
void orc_fr_from_std_vec(uint64_t* out, const uint64_t* in, size_t n);
void orc_fr_to_std(uint64_t s[4], const orc_fe* a);
void orc_fr_from_u64(orc_fe* r, uint64_t v);
void orc_fr_one(orc_fe* r);

/* ---- G1 (src/curve/g1.cuh) ---- */
void orc_g1_generator(orc_g1a* r);
void orc_g1_identity(orc_g1j* r);
void orc_g1_from_affine(orc_g1j* r, const orc_g1a* a);
void orc_g1_dbl(orc_g1j* r, const orc_g1j* a);
void orc_g1_add(orc_g1j* r, const orc_g1j* a, const orc_g1j* b);
void orc_g1_madd(orc_g1j* r, const orc_g1j* a, const orc_g1a* b);
void orc_g1_to_affine(orc_g1a* r, const orc_g1j* a);
void orc_g1_scalar_mul(orc_g1j* r, const orc_g1j* a, const orc_fe* s_mont);
int  orc_g1_is_on_curve(const orc_g1a* a);

/* ---- G2 (src/curve/g2.cuh) ---- */
void orc_g2_generator(orc_g2a* r);
void orc_g2_identity(orc_g2j* r);
void orc_g2_from_affine(orc_g2j* r, const orc_g2a* a);
void orc_g2_add_affine(orc_g2a* r, const orc_g2a* p, const orc_g2a* q);
void orc_g2_dbl_affine(orc_g2a* r, const orc_g2a* p);
void orc_g2_to_affine(orc_g2a* r, const orc_g2j* a);
void orc_g2_scalar_mul_affine(orc_g2a* r, const orc_g2a* p, const orc_fe* s_mont);
int  orc_g2_is_on_curve(const orc_g2a* a);

/* ---- MSM (src/msm/msm.cu:320-442 G1, :526-598 G2) ----
 * points: n affine records packed as x[4],y[4] (64 B); an all-zero record is
 * the point at infinity (never on the curve, since 0 != 3).  scalars: n Fr in
 * Montgomery form.  Result in affine; inf=1 for the identity.
 * nthreads <= 1 runs single-threaded; otherwise windows are split over threads. */
void orc_msm_g1(orc_g1a* out, const uint64_t* points64, const uint64_t* scalars, size_t n, int nthreads);
void orc_msm_g1_naive(orc_g1a* out, const uint64_t* points64, const uint64_t* scalars, size_t n);
void orc_msm_g2(orc_g2a* out, const uint64_t* points128, const uint64_t* scalars, size_t n, int nthreads);
void orc_msm_g2_naive(orc_g2a* out, const uint64_t* points128, const uint64_t* scalars, size_t n);
/* MSMConfig::for_size (src/msm/msm.cuh:46-63) */
void orc_msm_config(size_t n, int g2, int* window_bits, int* num_windows);

/* ---- NTT (src/ntt/ntt.cu) ---- */
void orc_compute_omega(orc_fe* r, int log_n, int inverse);
/* natural order in/out; inverse scales by n^-1; in and out may alias. */
void orc_ntt(uint64_t* out, const uint64_t* in, int log_n, int inverse);
/* the same transform with each stage split over nthreads threads */
void orc_ntt_mt(uint64_t* out, const uint64_t* in, int log_n, int inverse, int nthreads);
void orc_ntt_naive(uint64_t* out, const uint64_t* in, int log_n, int inverse);
/* coset forms used by compute_h (src/prover/groth16.cu:329-383):
 * coset forward  : out = NTT(a_i * g^i)
 * coset inverse  : out_i = INTT(a)_i * g^-i                               */
void orc_coset_ntt(uint64_t* out, const uint64_t* in, int log_n, int inverse, const orc_fe* g);
void orc_coset_ntt_mt(uint64_t* out, const uint64_t* in, int log_n, int inverse, const orc_fe* g, int nthreads);

/* ---- quotient polynomial (src/prover/groth16.cu:263-390) ----
 * Input: the three evaluation vectors A*w, B*w, C*w on the size-n domain.
 * Output: h coefficients (n entries).  Returns the coset generator used. */
void orc_compute_h_from_evals(uint64_t* h, const uint64_t* a_eval, const uint64_t* b_eval,
                              const uint64_t* c_eval, int log_n);

/* ---- helpers ---- */
/* mt19937_64 seeded generator matching std::mt19937_64 */
typedef struct { uint64_t mt[312]; int idx; } orc_rng;
void orc_rng_seed(orc_rng* r, uint64_t seed);
uint64_t orc_rng_next(orc_rng* r);
/* uniform Fr in Montgomery form: 4 draws, top limb masked to 254 bits, reject >= r */
void orc_rand_fr(orc_rng* r, orc_fe* out);
void orc_rand_fr_vec(orc_rng* r, uint64_t* out, size_t n);

/* ---- synthetic-input generators (test data, not on the reference path) ----
 * out_i = k_i * G for the group generator G, k_i Montgomery Fr scalars.
 * G1 uses a byte-comb table with Jacobian mixed additions; G2 uses Jacobian
 * formulas over Fp2 (a faster route to the same canonical affine points). */
void orc_g1_fixed_base(uint64_t* out64, const uint64_t* scalars, size_t n, int nthreads);
void orc_g2_fixed_base(uint64_t* out128, const uint64_t* scalars, size_t n, int nthreads);
int  orc_g2_is_on_curve_raw(const uint64_t* p128);

/* ---- full-size properties ----
 * sum_i a_i * b_i over Fr (Montgomery in, Montgomery out), multi-threaded;
 * with P_i = k_i G, MSM(P, s) = (sum_i s_i k_i) G for any size.            */
void orc_fr_dot(orc_fe* out, const uint64_t* a, const uint64_t* b, size_t n, int nthreads);
/* sum_i c_i x^i (Horner), i.e. one output of a forward NTT when x = w^k   */
void orc_fr_poly_eval(orc_fe* out, const uint64_t* coeffs, size_t n, const orc_fe* x);

#ifdef __cplusplus
}
#endif
#endif
