/*
 * bn254_oracle.c -- CPU restatement of cuda-zkml's Groth16 hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see bn254_oracle.h): the parity checker and the
 * timed CPU baseline.  Never linked into the product library.
 *
 * Only the curve definition (p, r, b = 3, the EIP-197 generators in standard
 * form) is written down here; every Montgomery constant (R, R^2, -m^-1, the
 * 2^28-th root of unity, 2^-1, the twist coefficient b') is derived at start-up
 * from first principles and compared against the reference's hard-coded values
 * by tests/test_oracle.py.
 */
#include "bn254_oracle.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

typedef unsigned __int128 u128;

/* ------------------------------------------------------------------ */
/* moduli                                                               */
/* ------------------------------------------------------------------ */
typedef struct {
    uint64_t m[4];
    uint64_t inv;   /* -m^-1 mod 2^64 */
    uint64_t one[4];/* R mod m */
    uint64_t r2[4]; /* R^2 mod m */
} modulus;

/* BN254 base field prime p (src/field/montgomery.cuh:33-38) */
static modulus MP = {{0x3C208C16D87CFD47ULL, 0x97816A916871CA8DULL, 0xB85045B68181585DULL, 0x30644E72E131A029ULL}, 0, {0}, {0}};
/* BN254 scalar field prime r (src/field/fp.cuh:330-335) */
static modulus MR = {{0x43E1F593F0000001ULL, 0x2833E84879B97091ULL, 0xB85045B68181585DULL, 0x30644E72E131A029ULL}, 0, {0}, {0}};

static int geq(const uint64_t a[4], const uint64_t b[4]) {
    for (int i = 3; i >= 0; i--) {
        if (a[i] != b[i]) return a[i] > b[i];
    }
    return 1;
}
static uint64_t add4(uint64_t r[4], const uint64_t a[4], const uint64_t b[4]) {
    u128 c = 0;
    for (int i = 0; i < 4; i++) { c += (u128)a[i] + b[i]; r[i] = (uint64_t)c; c >>= 64; }
    return (uint64_t)c;
}
static uint64_t sub4(uint64_t r[4], const uint64_t a[4], const uint64_t b[4]) {
    uint64_t br = 0;
    for (int i = 0; i < 4; i++) {
        u128 d = (u128)a[i] - b[i] - br;
        r[i] = (uint64_t)d;
        br = (uint64_t)(d >> 64) & 1;
    }
    return br;
}

/* modular add/sub for canonical inputs (< m) */
static void madd_(const modulus* M, uint64_t r[4], const uint64_t a[4], const uint64_t b[4]) {
    uint64_t t[4], u[4];
    uint64_t c = add4(t, a, b);
    uint64_t br = sub4(u, t, M->m);
    if (c || !br) memcpy(r, u, 32); else memcpy(r, t, 32);
}
static void msub_(const modulus* M, uint64_t r[4], const uint64_t a[4], const uint64_t b[4]) {
    uint64_t t[4];
    if (sub4(t, a, b)) add4(t, t, M->m);
    memcpy(r, t, 32);
}

/* CIOS Montgomery multiplication, 4 x 64-bit limbs (Koc, Acar, Kaliski 1996);
 * the same operand-scanning schedule as src/field/montgomery.cuh:306-348 with a
 * single final conditional subtraction.  Inputs < m give outputs < m. */
static void mmul_(const modulus* M, uint64_t r[4], const uint64_t a[4], const uint64_t b[4]) {
    uint64_t t[6] = {0, 0, 0, 0, 0, 0};
    for (int i = 0; i < 4; i++) {
        u128 c = 0;
        for (int j = 0; j < 4; j++) {
            c += (u128)a[i] * b[j] + t[j];
            t[j] = (uint64_t)c;
            c >>= 64;
        }
        c += t[4];
        t[4] = (uint64_t)c;
        t[5] = (uint64_t)(c >> 64);
        uint64_t mq = t[0] * M->inv;
        c = (u128)mq * M->m[0] + t[0];
        c >>= 64;
        for (int j = 1; j < 4; j++) {
            c += (u128)mq * M->m[j] + t[j];
            t[j - 1] = (uint64_t)c;
            c >>= 64;
        }
        c += t[4];
        t[3] = (uint64_t)c;
        t[4] = t[5] + (uint64_t)(c >> 64);
    }
    uint64_t u[4];
    uint64_t br = sub4(u, t, M->m);
    if (t[4] || !br) memcpy(r, u, 32); else memcpy(r, t, 32);
}

static void mpow_(const modulus* M, uint64_t r[4], const uint64_t a[4], const uint64_t e[4]) {
    uint64_t acc[4], base[4];
    memcpy(acc, M->one, 32);
    memcpy(base, a, 32);
    for (int bit = 255; bit >= 0; bit--) {
        mmul_(M, acc, acc, acc);
        if ((e[bit >> 6] >> (bit & 63)) & 1) mmul_(M, acc, acc, base);
    }
    memcpy(r, acc, 32);
}

/* Fermat inverse a^(m-2) (src/field/fp.cuh:257-266, :556-564) */
static void minv_(const modulus* M, uint64_t r[4], const uint64_t a[4]) {
    uint64_t e[4], two[4] = {2, 0, 0, 0};
    sub4(e, M->m, two);
    mpow_(M, r, a, e);
}

static void derive_modulus(modulus* M) {
    /* -m^-1 mod 2^64 by Newton iteration x <- x(2 - m x) */
    uint64_t x = 1;
    for (int i = 0; i < 7; i++) x = x * (2 - M->m[0] * x);
    M->inv = (uint64_t)(0 - x);
    /* R mod m = 2^256 mod m by 256 modular doublings of 1 */
    uint64_t v[4] = {1, 0, 0, 0};
    for (int i = 0; i < 256; i++) madd_(M, v, v, v);
    memcpy(M->one, v, 32);
    for (int i = 0; i < 256; i++) madd_(M, v, v, v);
    memcpy(M->r2, v, 32);
}

/* ------------------------------------------------------------------ */
/* derived constants                                                    */
/* ------------------------------------------------------------------ */
static orc_fe OMEGA28, OMEGA28_INV, FR_HALF, G2_B;
static orc_fe2 G2_B2;
static orc_g2a G2_GEN;
static pthread_once_t g_once = PTHREAD_ONCE_INIT;

/* EIP-197 G2 generator, standard form (the decimal values quoted in
 * src/curve/g2.cuh:8-13). */
static const uint64_t G2X0[4] = {0x46DEBD5CD992F6EDULL, 0x674322D4F75EDADDULL, 0x426A00665E5C4479ULL, 0x1800DEEF121F1E76ULL};
static const uint64_t G2X1[4] = {0x97E485B7AEF312C2ULL, 0xF1AA493335A9E712ULL, 0x7260BFB731FB5D25ULL, 0x198E9393920D483AULL};
static const uint64_t G2Y0[4] = {0x4CE6CC0166FA7DAAULL, 0xE3D1E7690C43D37BULL, 0x4AAB71808DCB408FULL, 0x12C85EA5DB8C6DEBULL};
static const uint64_t G2Y1[4] = {0x55ACDADCD122975BULL, 0xBC4B313370B38EF3ULL, 0xEC9E99AD690C3395ULL, 0x090689D0585FF075ULL};

static void init_once(void) {
    derive_modulus(&MP);
    derive_modulus(&MR);
    /* omega_{2^28} = 5^((r-1)/2^28) mod r (src/ntt/ntt.cu:43-62) */
    uint64_t e[4], one[4] = {1, 0, 0, 0}, five[4] = {5, 0, 0, 0};
    sub4(e, MR.m, one);
    for (int s = 0; s < 28; s++) { /* e >>= 1 */
        for (int i = 0; i < 4; i++) e[i] = (e[i] >> 1) | (i < 3 ? e[i + 1] << 63 : 0);
    }
    uint64_t g[4];
    mmul_(&MR, g, five, MR.r2);
    mpow_(&MR, OMEGA28.v, g, e);
    minv_(&MR, OMEGA28_INV.v, OMEGA28.v);
    /* 2^-1 mod r in Montgomery form (src/ntt/ntt.cu:437-451) */
    uint64_t two[4] = {2, 0, 0, 0}, t2[4];
    mmul_(&MR, t2, two, MR.r2);
    minv_(&MR, FR_HALF.v, t2);
    /* twist coefficient b' = 3 / (9 + u) (src/curve/g2.cuh:35-44) */
    orc_fe three, nine, zero;
    memset(&zero, 0, sizeof zero);
    uint64_t s3[4] = {3, 0, 0, 0}, s9[4] = {9, 0, 0, 0};
    mmul_(&MP, three.v, s3, MP.r2);
    mmul_(&MP, nine.v, s9, MP.r2);
    /* 1/(9+u) = (9-u)/(81+1) */
    orc_fe nrm, nrm_inv, t;
    mmul_(&MP, nrm.v, nine.v, nine.v);
    madd_(&MP, nrm.v, nrm.v, MP.one);
    minv_(&MP, nrm_inv.v, nrm.v);
    mmul_(&MP, t.v, nine.v, nrm_inv.v);
    mmul_(&MP, G2_B2.c0.v, t.v, three.v);
    mmul_(&MP, t.v, MP.one, nrm_inv.v);
    msub_(&MP, t.v, zero.v, t.v);
    mmul_(&MP, G2_B2.c1.v, t.v, three.v);
    G2_B = G2_B2.c0;
    mmul_(&MP, G2_GEN.x.c0.v, G2X0, MP.r2);
    mmul_(&MP, G2_GEN.x.c1.v, G2X1, MP.r2);
    mmul_(&MP, G2_GEN.y.c0.v, G2Y0, MP.r2);
    mmul_(&MP, G2_GEN.y.c1.v, G2Y1, MP.r2);
    G2_GEN.inf = 0;
}
#define INIT() pthread_once(&g_once, init_once)

/* ------------------------------------------------------------------ */
/* Fp / Fr public wrappers                                              */
/* ------------------------------------------------------------------ */
void orc_fp_mul(orc_fe* r, const orc_fe* a, const orc_fe* b) { INIT(); mmul_(&MP, r->v, a->v, b->v); }
void orc_fp_add(orc_fe* r, const orc_fe* a, const orc_fe* b) { INIT(); madd_(&MP, r->v, a->v, b->v); }
void orc_fp_sub(orc_fe* r, const orc_fe* a, const orc_fe* b) { INIT(); msub_(&MP, r->v, a->v, b->v); }
void orc_fp_neg(orc_fe* r, const orc_fe* a) { orc_fe z; memset(&z, 0, sizeof z); orc_fp_sub(r, &z, a); }
void orc_fp_inv(orc_fe* r, const orc_fe* a) { INIT(); minv_(&MP, r->v, a->v); }
void orc_fp_from_std(orc_fe* r, const uint64_t s[4]) { INIT(); mmul_(&MP, r->v, s, MP.r2); }
void orc_fp_to_std(uint64_t s[4], const orc_fe* a) { INIT(); uint64_t one[4] = {1, 0, 0, 0}; mmul_(&MP, s, a->v, one); }
void orc_fp_one(orc_fe* r) { INIT(); memcpy(r->v, MP.one, 32); }

void orc_fr_mul(orc_fe* r, const orc_fe* a, const orc_fe* b) { INIT(); mmul_(&MR, r->v, a->v, b->v); }
void orc_fr_add(orc_fe* r, const orc_fe* a, const orc_fe* b) { INIT(); madd_(&MR, r->v, a->v, b->v); }
void orc_fr_sub(orc_fe* r, const orc_fe* a, const orc_fe* b) { INIT(); msub_(&MR, r->v, a->v, b->v); }
void orc_fr_inv(orc_fe* r, const orc_fe* a) { INIT(); minv_(&MR, r->v, a->v); }
void orc_fr_from_std(orc_fe* r, const uint64_t s[4]) { INIT(); mmul_(&MR, r->v, s, MR.r2); }
void orc_fr_from_std_vec(uint64_t* out, const uint64_t* in, size_t n) {
    INIT();
    for (size_t i = 0; i < n; i++) mmul_(&MR, out + 4 * i, in + 4 * i, MR.r2);
}
void orc_fr_to_std(uint64_t s[4], const orc_fe* a) { INIT(); uint64_t one[4] = {1, 0, 0, 0}; mmul_(&MR, s, a->v, one); }
void orc_fr_from_u64(orc_fe* r, uint64_t v) { uint64_t s[4] = {v, 0, 0, 0}; orc_fr_from_std(r, s); }
void orc_fr_one(orc_fe* r) { INIT(); memcpy(r->v, MR.one, 32); }

static int fe_is_zero(const orc_fe* a) { return (a->v[0] | a->v[1] | a->v[2] | a->v[3]) == 0; }
static int fe_eq(const orc_fe* a, const orc_fe* b) { return memcmp(a, b, 32) == 0; }

/* short internal Fp helpers (constants initialised by the caller) */
static inline void FM(orc_fe* r, const orc_fe* a, const orc_fe* b) { mmul_(&MP, r->v, a->v, b->v); }
static inline void FA(orc_fe* r, const orc_fe* a, const orc_fe* b) { madd_(&MP, r->v, a->v, b->v); }
static inline void FS(orc_fe* r, const orc_fe* a, const orc_fe* b) { msub_(&MP, r->v, a->v, b->v); }

/* ------------------------------------------------------------------ */
/* G1: y^2 = x^3 + 3, Jacobian coordinates (src/curve/g1.cuh)           */
/* ------------------------------------------------------------------ */
void orc_g1_generator(orc_g1a* r) {
    INIT();
    uint64_t one[4] = {1, 0, 0, 0}, two[4] = {2, 0, 0, 0};
    mmul_(&MP, r->x.v, one, MP.r2);
    mmul_(&MP, r->y.v, two, MP.r2);
    r->inf = 0;
}
void orc_g1_identity(orc_g1j* r) { INIT(); memset(r, 0, sizeof *r); memcpy(r->y.v, MP.one, 32); }
void orc_g1_from_affine(orc_g1j* r, const orc_g1a* a) {
    if (a->inf) { orc_g1_identity(r); return; }
    INIT();
    r->x = a->x; r->y = a->y; memcpy(r->z.v, MP.one, 32);
}

/* dbl-2009-l (src/curve/g1.cuh:89-117) */
void orc_g1_dbl(orc_g1j* r, const orc_g1j* p) {
    INIT();
    if (fe_is_zero(&p->z)) { *r = *p; return; }
    orc_fe A, B, C, D, E, F, X3, Y3, Z3, t, C8, zz;
    FM(&A, &p->x, &p->x);
    FM(&B, &p->y, &p->y);
    FM(&C, &B, &B);
    FA(&t, &p->x, &B); FM(&D, &t, &t); FS(&D, &D, &A); FS(&D, &D, &C); FA(&D, &D, &D);
    FA(&E, &A, &A); FA(&E, &E, &A);
    FM(&F, &E, &E);
    FS(&X3, &F, &D); FS(&X3, &X3, &D);
    FA(&C8, &C, &C); FA(&C8, &C8, &C8); FA(&C8, &C8, &C8);
    FS(&t, &D, &X3); FM(&Y3, &E, &t); FS(&Y3, &Y3, &C8);
    FA(&t, &p->y, &p->z); FM(&Z3, &t, &t); FS(&Z3, &Z3, &B); FM(&zz, &p->z, &p->z); FS(&Z3, &Z3, &zz);
    r->x = X3; r->y = Y3; r->z = Z3;
}

/* full Jacobian addition (src/curve/g1.cuh:121-159) */
void orc_g1_add(orc_g1j* r, const orc_g1j* p, const orc_g1j* q) {
    INIT();
    if (fe_is_zero(&p->z)) { *r = *q; return; }
    if (fe_is_zero(&q->z)) { *r = *p; return; }
    orc_fe Z1Z1, Z2Z2, U1, U2, S1, S2, H, R, HH, HHH, V, X3, Y3, Z3, t;
    FM(&Z1Z1, &p->z, &p->z);
    FM(&Z2Z2, &q->z, &q->z);
    FM(&U1, &p->x, &Z2Z2);
    FM(&U2, &q->x, &Z1Z1);
    FM(&t, &p->y, &q->z); FM(&S1, &t, &Z2Z2);
    FM(&t, &q->y, &p->z); FM(&S2, &t, &Z1Z1);
    FS(&H, &U2, &U1);
    FS(&R, &S2, &S1);
    if (fe_is_zero(&H)) {
        if (fe_is_zero(&R)) { orc_g1_dbl(r, p); return; }
        orc_g1_identity(r); return;
    }
    FM(&HH, &H, &H);
    FM(&HHH, &HH, &H);
    FM(&V, &U1, &HH);
    FM(&X3, &R, &R); FS(&X3, &X3, &HHH); FS(&X3, &X3, &V); FS(&X3, &X3, &V);
    FS(&t, &V, &X3); FM(&Y3, &R, &t); FM(&t, &S1, &HHH); FS(&Y3, &Y3, &t);
    FM(&t, &p->z, &q->z); FM(&Z3, &t, &H);
    r->x = X3; r->y = Y3; r->z = Z3;
}

/* mixed Jacobian + affine addition (src/curve/g1.cuh:163-189) */
void orc_g1_madd(orc_g1j* r, const orc_g1j* p, const orc_g1a* q) {
    INIT();
    if (q->inf) { *r = *p; return; }
    if (fe_is_zero(&p->z)) { orc_g1_from_affine(r, q); return; }
    orc_fe Z1Z1, U2, S2, H, R, HH, HHH, V, X3, Y3, Z3, t;
    FM(&Z1Z1, &p->z, &p->z);
    FM(&U2, &q->x, &Z1Z1);
    FM(&t, &q->y, &p->z); FM(&S2, &t, &Z1Z1);
    FS(&H, &U2, &p->x);
    FS(&R, &S2, &p->y);
    if (fe_is_zero(&H)) {
        if (fe_is_zero(&R)) { orc_g1_dbl(r, p); return; }
        orc_g1_identity(r); return;
    }
    FM(&HH, &H, &H);
    FM(&HHH, &HH, &H);
    FM(&V, &p->x, &HH);
    FM(&X3, &R, &R); FS(&X3, &X3, &HHH); FS(&X3, &X3, &V); FS(&X3, &X3, &V);
    FS(&t, &V, &X3); FM(&Y3, &R, &t); FM(&t, &p->y, &HHH); FS(&Y3, &Y3, &t);
    FM(&Z3, &p->z, &H);
    r->x = X3; r->y = Y3; r->z = Z3;
}

/* src/curve/g1.cuh:78-84 */
void orc_g1_to_affine(orc_g1a* r, const orc_g1j* p) {
    INIT();
    if (fe_is_zero(&p->z)) { memset(r, 0, sizeof *r); r->inf = 1; return; }
    orc_fe zi, zi2, zi3;
    minv_(&MP, zi.v, p->z.v);
    FM(&zi2, &zi, &zi);
    FM(&zi3, &zi2, &zi);
    FM(&r->x, &p->x, &zi2);
    FM(&r->y, &p->y, &zi3);
    r->inf = 0;
}

/* double-and-add from the top bit of the standard-form scalar (g1.cuh:204-246) */
void orc_g1_scalar_mul(orc_g1j* r, const orc_g1j* p, const orc_fe* s_mont) {
    uint64_t s[4];
    orc_fr_to_std(s, s_mont);
    orc_g1j acc;
    orc_g1_identity(&acc);
    for (int bit = 255; bit >= 0; bit--) {
        orc_g1_dbl(&acc, &acc);
        if ((s[bit >> 6] >> (bit & 63)) & 1) orc_g1_add(&acc, &acc, p);
    }
    *r = acc;
}

int orc_g1_is_on_curve(const orc_g1a* a) {
    INIT();
    if (a->inf) return 1;
    orc_fe y2, x3, b;
    uint64_t s3[4] = {3, 0, 0, 0};
    mmul_(&MP, b.v, s3, MP.r2);
    FM(&y2, &a->y, &a->y);
    FM(&x3, &a->x, &a->x); FM(&x3, &x3, &a->x); FA(&x3, &x3, &b);
    return fe_eq(&y2, &x3);
}

/* ------------------------------------------------------------------ */
/* Fp2 and G2 (src/field/fp2.cuh, src/curve/g2.cuh)                     */
/* ------------------------------------------------------------------ */
static void f2_add(orc_fe2* r, const orc_fe2* a, const orc_fe2* b) { FA(&r->c0, &a->c0, &b->c0); FA(&r->c1, &a->c1, &b->c1); }
static void f2_sub(orc_fe2* r, const orc_fe2* a, const orc_fe2* b) { FS(&r->c0, &a->c0, &b->c0); FS(&r->c1, &a->c1, &b->c1); }
/* Karatsuba, fp2.cuh:73-78 */
static void f2_mul(orc_fe2* r, const orc_fe2* a, const orc_fe2* b) {
    orc_fe ac, bd, s1, s2, m;
    FM(&ac, &a->c0, &b->c0);
    FM(&bd, &a->c1, &b->c1);
    FA(&s1, &a->c0, &a->c1);
    FA(&s2, &b->c0, &b->c1);
    FM(&m, &s1, &s2);
    FS(&r->c0, &ac, &bd);
    FS(&m, &m, &ac);
    FS(&r->c1, &m, &bd);
}
static void f2_sqr(orc_fe2* r, const orc_fe2* a) { f2_mul(r, a, a); }
/* inverse via the norm, fp2.cuh:110-114 */
static void f2_inv(orc_fe2* r, const orc_fe2* a) {
    orc_fe n, t, ni, z;
    memset(&z, 0, sizeof z);
    FM(&n, &a->c0, &a->c0); FM(&t, &a->c1, &a->c1); FA(&n, &n, &t);
    minv_(&MP, ni.v, n.v);
    FM(&r->c0, &a->c0, &ni);
    FM(&t, &a->c1, &ni);
    FS(&r->c1, &z, &t);
}
static int f2_is_zero(const orc_fe2* a) { return fe_is_zero(&a->c0) && fe_is_zero(&a->c1); }
static int f2_eq(const orc_fe2* a, const orc_fe2* b) { return fe_eq(&a->c0, &b->c0) && fe_eq(&a->c1, &b->c1); }
static void f2_one(orc_fe2* r) { memset(r, 0, sizeof *r); memcpy(r->c0.v, MP.one, 32); }

void orc_g2_generator(orc_g2a* r) { INIT(); *r = G2_GEN; }
void orc_g2_identity(orc_g2j* r) { INIT(); memset(r, 0, sizeof *r); f2_one(&r->y); }
void orc_g2_from_affine(orc_g2j* r, const orc_g2a* a) {
    if (a->inf) { orc_g2_identity(r); return; }
    INIT();
    r->x = a->x; r->y = a->y; f2_one(&r->z);
}
/* affine doubling, g2.cuh:103-116 */
void orc_g2_dbl_affine(orc_g2a* r, const orc_g2a* p) {
    INIT();
    if (p->inf || f2_is_zero(&p->y)) { memset(r, 0, sizeof *r); r->inf = 1; return; }
    orc_fe2 num, den, lam, t, x3, y3;
    f2_sqr(&t, &p->x);
    f2_add(&num, &t, &t); f2_add(&num, &num, &t);       /* 3 x^2 */
    f2_add(&den, &p->y, &p->y);                          /* 2 y */
    f2_inv(&t, &den); f2_mul(&lam, &num, &t);
    f2_sqr(&x3, &lam); f2_sub(&x3, &x3, &p->x); f2_sub(&x3, &x3, &p->x);
    f2_sub(&t, &p->x, &x3); f2_mul(&y3, &lam, &t); f2_sub(&y3, &y3, &p->y);
    r->x = x3; r->y = y3; r->inf = 0;
}
/* affine addition, g2.cuh:118-131 */
void orc_g2_add_affine(orc_g2a* r, const orc_g2a* p, const orc_g2a* q) {
    INIT();
    if (p->inf) { *r = *q; return; }
    if (q->inf) { *r = *p; return; }
    if (f2_eq(&p->x, &q->x)) {
        if (!f2_eq(&p->y, &q->y)) { memset(r, 0, sizeof *r); r->inf = 1; return; }
        orc_g2_dbl_affine(r, p); return;
    }
    orc_fe2 num, den, lam, t, x3, y3;
    f2_sub(&num, &q->y, &p->y);
    f2_sub(&den, &q->x, &p->x);
    f2_inv(&t, &den); f2_mul(&lam, &num, &t);
    f2_sqr(&x3, &lam); f2_sub(&x3, &x3, &p->x); f2_sub(&x3, &x3, &q->x);
    f2_sub(&t, &p->x, &x3); f2_mul(&y3, &lam, &t); f2_sub(&y3, &y3, &p->y);
    r->x = x3; r->y = y3; r->inf = 0;
}
void orc_g2_to_affine(orc_g2a* r, const orc_g2j* p) {
    INIT();
    if (f2_is_zero(&p->z)) { memset(r, 0, sizeof *r); r->inf = 1; return; }
    orc_fe2 zi, zi2, zi3;
    f2_inv(&zi, &p->z);
    f2_sqr(&zi2, &zi);
    f2_mul(&zi3, &zi2, &zi);
    f2_mul(&r->x, &p->x, &zi2);
    f2_mul(&r->y, &p->y, &zi3);
    r->inf = 0;
}
void orc_g2_scalar_mul_affine(orc_g2a* r, const orc_g2a* p, const orc_fe* s_mont) {
    uint64_t s[4];
    orc_fr_to_std(s, s_mont);
    orc_g2a acc;
    memset(&acc, 0, sizeof acc); acc.inf = 1;
    for (int bit = 255; bit >= 0; bit--) {
        orc_g2_dbl_affine(&acc, &acc);
        if ((s[bit >> 6] >> (bit & 63)) & 1) orc_g2_add_affine(&acc, &acc, p);
    }
    *r = acc;
}
int orc_g2_is_on_curve(const orc_g2a* a) {
    INIT();
    if (a->inf) return 1;
    orc_fe2 y2, x3;
    f2_sqr(&y2, &a->y);
    f2_sqr(&x3, &a->x); f2_mul(&x3, &x3, &a->x); f2_add(&x3, &x3, &G2_B2);
    return f2_eq(&y2, &x3);
}

/* ------------------------------------------------------------------ */
/* MSM (src/msm/msm.cu)                                                  */
/* ------------------------------------------------------------------ */
/* MSMConfig::for_size (src/msm/msm.cuh:46-63); G2 caps c at 12 (msm.cu:529-533) */
void orc_msm_config(size_t n, int g2, int* window_bits, int* num_windows) {
    int c;
    if (n <= (1u << 10)) c = 10;
    else if (n <= (1u << 14)) c = 12;
    else if (n <= (1u << 18)) c = 14;
    else if (n <= (1u << 22)) c = 15;
    else c = 16;
    if (g2 && c > 12) c = 12;
    *window_bits = c;
    *num_windows = (253 + c) / c;
}

/* unsigned c-bit window of a standard-form scalar (msm.cu:124-142) */
static uint32_t window_digit(const uint64_t s[4], int w, int c) {
    int off = w * c, limb = off >> 6, sh = off & 63;
    uint64_t mask = ((uint64_t)1 << c) - 1;
    if (limb >= 4) return 0;
    uint64_t v = s[limb] >> sh;
    if (sh + c > 64 && limb + 1 < 4) v |= s[limb + 1] << (64 - sh);
    return (uint32_t)(v & mask);
}

static int g1_point_is_inf(const uint64_t* p64) {
    for (int i = 0; i < 8; i++) if (p64[i]) return 0;
    return 1;
}

typedef struct {
    const uint64_t* pts;
    const uint64_t* std_scalars;
    size_t n;
    int c, w0, w1;
    orc_g1j* window_out;
} g1_job;

/* Per window: bucket accumulate with mixed adds, then the reverse running
 * sum (msm.cu:104-154, :284-307). */
static void* g1_window_worker(void* arg) {
    g1_job* J = (g1_job*)arg;
    size_t nb = ((size_t)1 << J->c) - 1;
    orc_g1j* buckets = (orc_g1j*)malloc(nb * sizeof(orc_g1j));
    for (int w = J->w0; w < J->w1; w++) {
        for (size_t b = 0; b < nb; b++) orc_g1_identity(&buckets[b]);
        for (size_t i = 0; i < J->n; i++) {
            const uint64_t* p = J->pts + 8 * i;
            if (g1_point_is_inf(p)) continue;
            uint32_t d = window_digit(J->std_scalars + 4 * i, w, J->c);
            if (!d) continue;
            orc_g1a a;
            memcpy(a.x.v, p, 32); memcpy(a.y.v, p + 4, 32); a.inf = 0;
            orc_g1_madd(&buckets[d - 1], &buckets[d - 1], &a);
        }
        orc_g1j run, sum;
        orc_g1_identity(&run); orc_g1_identity(&sum);
        for (size_t b = nb; b-- > 0;) {
            if (!fe_is_zero(&buckets[b].z)) orc_g1_add(&run, &run, &buckets[b]);
            orc_g1_add(&sum, &sum, &run);
        }
        J->window_out[w] = sum;
    }
    free(buckets);
    return NULL;
}

void orc_msm_g1(orc_g1a* out, const uint64_t* points64, const uint64_t* scalars, size_t n, int nthreads) {
    INIT();
    orc_g1j res;
    orc_g1_identity(&res);
    if (n == 0) { orc_g1_to_affine(out, &res); return; }
    int c, W;
    orc_msm_config(n, 0, &c, &W);
    uint64_t* st = (uint64_t*)malloc(n * 32);
    for (size_t i = 0; i < n; i++) orc_fr_to_std(st + 4 * i, (const orc_fe*)(scalars + 4 * i));
    orc_g1j* wins = (orc_g1j*)malloc(W * sizeof(orc_g1j));
    if (nthreads < 1) nthreads = 1;
    if (nthreads > W) nthreads = W;
    pthread_t* th = (pthread_t*)malloc(nthreads * sizeof(pthread_t));
    g1_job* jobs = (g1_job*)malloc(nthreads * sizeof(g1_job));
    for (int t = 0; t < nthreads; t++) {
        jobs[t].pts = points64; jobs[t].std_scalars = st; jobs[t].n = n; jobs[t].c = c;
        jobs[t].w0 = (int)((long)W * t / nthreads); jobs[t].w1 = (int)((long)W * (t + 1) / nthreads);
        jobs[t].window_out = wins;
        if (nthreads == 1) g1_window_worker(&jobs[t]);
        else pthread_create(&th[t], NULL, g1_window_worker, &jobs[t]);
    }
    if (nthreads > 1) for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
    /* window combine on the host (msm.cu:423-430) */
    for (int w = W - 1; w >= 0; w--) {
        for (int i = 0; i < c; i++) orc_g1_dbl(&res, &res);
        orc_g1_add(&res, &res, &wins[w]);
    }
    orc_g1_to_affine(out, &res);
    free(st); free(wins); free(th); free(jobs);
}

/* sum of per-point scalar multiplications: the reference's small-n path
 * (msm.cu:330-339) and its test oracle cpu_msm (tests/test_msm.cu:20-28) */
void orc_msm_g1_naive(orc_g1a* out, const uint64_t* points64, const uint64_t* scalars, size_t n) {
    orc_g1j res, t, p;
    orc_g1_identity(&res);
    for (size_t i = 0; i < n; i++) {
        orc_g1a a;
        memcpy(a.x.v, points64 + 8 * i, 32); memcpy(a.y.v, points64 + 8 * i + 4, 32);
        a.inf = g1_point_is_inf(points64 + 8 * i);
        orc_g1_from_affine(&p, &a);
        orc_g1_scalar_mul(&t, &p, (const orc_fe*)(scalars + 4 * i));
        orc_g1_add(&res, &res, &t);
    }
    orc_g1_to_affine(out, &res);
}

static void g2_load(orc_g2a* a, const uint64_t* p) {
    memcpy(a->x.c0.v, p, 32); memcpy(a->x.c1.v, p + 4, 32);
    memcpy(a->y.c0.v, p + 8, 32); memcpy(a->y.c1.v, p + 12, 32);
    a->inf = 1;
    for (int i = 0; i < 16; i++) if (p[i]) { a->inf = 0; break; }
}

typedef struct {
    const uint64_t* pts;
    const uint64_t* std_scalars;
    size_t n;
    int c, w0, w1;
    orc_g2a* window_out;
} g2_job;

/* G2 buckets: every G2 operation in the reference goes through affine
 * coordinates with an Fp2 inversion (g2.cuh:134-146), so the buckets are kept
 * affine here. */
static void* g2_window_worker(void* arg) {
    g2_job* J = (g2_job*)arg;
    size_t nb = ((size_t)1 << J->c) - 1;
    orc_g2a* buckets = (orc_g2a*)malloc(nb * sizeof(orc_g2a));
    for (int w = J->w0; w < J->w1; w++) {
        for (size_t b = 0; b < nb; b++) { memset(&buckets[b], 0, sizeof(orc_g2a)); buckets[b].inf = 1; }
        for (size_t i = 0; i < J->n; i++) {
            orc_g2a a;
            g2_load(&a, J->pts + 16 * i);
            if (a.inf) continue;
            uint32_t d = window_digit(J->std_scalars + 4 * i, w, J->c);
            if (!d) continue;
            orc_g2_add_affine(&buckets[d - 1], &buckets[d - 1], &a);
        }
        orc_g2a run, sum;
        memset(&run, 0, sizeof run); run.inf = 1; sum = run;
        for (size_t b = nb; b-- > 0;) {
            orc_g2_add_affine(&run, &run, &buckets[b]);
            orc_g2_add_affine(&sum, &sum, &run);
        }
        J->window_out[w] = sum;
    }
    free(buckets);
    return NULL;
}

void orc_msm_g2(orc_g2a* out, const uint64_t* points128, const uint64_t* scalars, size_t n, int nthreads) {
    INIT();
    orc_g2a res;
    memset(&res, 0, sizeof res); res.inf = 1;
    if (n == 0) { *out = res; return; }
    int c, W;
    orc_msm_config(n, 1, &c, &W);
    uint64_t* st = (uint64_t*)malloc(n * 32);
    for (size_t i = 0; i < n; i++) orc_fr_to_std(st + 4 * i, (const orc_fe*)(scalars + 4 * i));
    orc_g2a* wins = (orc_g2a*)malloc(W * sizeof(orc_g2a));
    if (nthreads < 1) nthreads = 1;
    if (nthreads > W) nthreads = W;
    pthread_t* th = (pthread_t*)malloc(nthreads * sizeof(pthread_t));
    g2_job* jobs = (g2_job*)malloc(nthreads * sizeof(g2_job));
    for (int t = 0; t < nthreads; t++) {
        jobs[t].pts = points128; jobs[t].std_scalars = st; jobs[t].n = n; jobs[t].c = c;
        jobs[t].w0 = (int)((long)W * t / nthreads); jobs[t].w1 = (int)((long)W * (t + 1) / nthreads);
        jobs[t].window_out = wins;
        if (nthreads == 1) g2_window_worker(&jobs[t]);
        else pthread_create(&th[t], NULL, g2_window_worker, &jobs[t]);
    }
    if (nthreads > 1) for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
    for (int w = W - 1; w >= 0; w--) {
        for (int i = 0; i < c; i++) orc_g2_dbl_affine(&res, &res);
        orc_g2_add_affine(&res, &res, &wins[w]);
    }
    *out = res;
    free(st); free(wins); free(th); free(jobs);
}

void orc_msm_g2_naive(orc_g2a* out, const uint64_t* points128, const uint64_t* scalars, size_t n) {
    orc_g2a res, t, a;
    memset(&res, 0, sizeof res); res.inf = 1;
    for (size_t i = 0; i < n; i++) {
        g2_load(&a, points128 + 16 * i);
        orc_g2_scalar_mul_affine(&t, &a, (const orc_fe*)(scalars + 4 * i));
        orc_g2_add_affine(&res, &res, &t);
    }
    *out = res;
}

/* ------------------------------------------------------------------ */
/* NTT (src/ntt/ntt.cu)                                                  */
/* ------------------------------------------------------------------ */
/* omega_{2^log_n} = omega_{2^28}^(2^(28-log_n)) (ntt.cu:64-106) */
void orc_compute_omega(orc_fe* r, int log_n, int inverse) {
    INIT();
    orc_fe w = inverse ? OMEGA28_INV : OMEGA28;
    for (int i = 0; i < 28 - log_n; i++) mmul_(&MR, w.v, w.v, w.v);
    *r = w;
}

static uint32_t bitrev(uint32_t x, int bits) {
    uint32_t r = 0;
    for (int i = 0; i < bits; i++) { r = (r << 1) | (x & 1); x >>= 1; }
    return r;
}

/* bit-reverse, radix-2 DIT stages with t = w^(pos << (log_n-1-s)) * b,
 * (a+t, a-t), then the n^-1 scale for the inverse (ntt.cu:354-465).
 * The multi-threaded form splits each stage's butterflies (and the stage's
 * twiddle table) into contiguous ranges: every value is computed exactly as in
 * the single-threaded loop. */
typedef struct {
    uint64_t* buf; const uint64_t* in; orc_fe* tw; orc_fe ws; orc_fe sc;
    size_t n, lo, hi; int log_n, stage, phase;
} ntt_job;

static void ntt_job_run(ntt_job* J) {
    const size_t stride = (size_t)1 << J->stage;
    if (J->phase == 0) {          /* bit-reversed copy of elements [lo, hi) */
        for (size_t i = J->lo; i < J->hi; i++) memcpy(J->buf + 4 * bitrev((uint32_t)i, J->log_n), J->in + 4 * i, 32);
    } else if (J->phase == 1) {   /* twiddles tw[k] = ws^k, k in [lo, hi) */
        uint64_t e[4] = {J->lo, 0, 0, 0};
        mpow_(&MR, J->tw[J->lo].v, J->ws.v, e);
        for (size_t k = J->lo + 1; k < J->hi; k++) mmul_(&MR, J->tw[k].v, J->tw[k - 1].v, J->ws.v);
    } else if (J->phase == 2) {   /* butterflies j in [lo, hi): group j / stride, offset j % stride */
        for (size_t j = J->lo; j < J->hi; j++) {
            const size_t k = j & (stride - 1), g = (j >> J->stage) << (J->stage + 1);
            uint64_t* a = J->buf + 4 * (g + k);
            uint64_t* b = J->buf + 4 * (g + k + stride);
            uint64_t t[4], s0[4];
            mmul_(&MR, t, J->tw[k].v, b);
            madd_(&MR, s0, a, t);
            msub_(&MR, b, a, t);
            memcpy(a, s0, 32);
        }
    } else {                      /* n^-1 scale of [lo, hi) */
        for (size_t i = J->lo; i < J->hi; i++) mmul_(&MR, J->buf + 4 * i, J->buf + 4 * i, J->sc.v);
    }
}

static void* ntt_worker(void* arg) { ntt_job_run((ntt_job*)arg); return NULL; }

/* run `proto` over [0, count) split into nthreads ranges */
static void ntt_parallel(const ntt_job* proto, size_t count, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if ((size_t)nthreads > count) nthreads = count ? (int)count : 1;
    if (nthreads == 1 || count < 4096) {
        ntt_job J = *proto;
        J.lo = 0; J.hi = count;
        ntt_job_run(&J);
        return;
    }
    pthread_t th[256];
    ntt_job jobs[256];
    if (nthreads > 256) nthreads = 256;
    for (int t = 0; t < nthreads; t++) {
        jobs[t] = *proto;
        jobs[t].lo = count * t / nthreads;
        jobs[t].hi = count * (t + 1) / nthreads;
        pthread_create(&th[t], NULL, ntt_worker, &jobs[t]);
    }
    for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
}

void orc_ntt_mt(uint64_t* out, const uint64_t* in, int log_n, int inverse, int nthreads) {
    INIT();
    size_t n = (size_t)1 << log_n;
    uint64_t* buf = (uint64_t*)malloc(n * 32);
    orc_fe* tw = (orc_fe*)malloc((n / 2 + 1) * sizeof(orc_fe));
    ntt_job P;
    memset(&P, 0, sizeof P);
    P.buf = buf; P.in = in; P.tw = tw; P.n = n; P.log_n = log_n;
    P.phase = 0;
    ntt_parallel(&P, n, nthreads);
    orc_fe w;
    orc_compute_omega(&w, log_n, inverse);
    for (int s = 0; s < log_n; s++) {
        orc_fe ws = w;
        for (int i = 0; i < log_n - 1 - s; i++) mmul_(&MR, ws.v, ws.v, ws.v);
        P.stage = s;
        P.ws = ws;
        P.phase = 1;
        ntt_parallel(&P, (size_t)1 << s, nthreads);
        P.phase = 2;
        ntt_parallel(&P, n / 2, nthreads);
    }
    if (inverse) {
        memcpy(P.sc.v, MR.one, 32);
        for (int i = 0; i < log_n; i++) mmul_(&MR, P.sc.v, P.sc.v, FR_HALF.v);
        P.phase = 3;
        ntt_parallel(&P, n, nthreads);
    }
    memcpy(out, buf, n * 32);
    free(buf); free(tw);
}

void orc_ntt(uint64_t* out, const uint64_t* in, int log_n, int inverse) { orc_ntt_mt(out, in, log_n, inverse, 1); }

/* O(n^2) DFT, tests/test_ntt.cu:19-37 */
void orc_ntt_naive(uint64_t* out, const uint64_t* in, int log_n, int inverse) {
    INIT();
    size_t n = (size_t)1 << log_n;
    orc_fe w, wi, wij, acc, t;
    orc_compute_omega(&w, log_n, inverse);
    uint64_t* buf = (uint64_t*)malloc(n * 32);
    memcpy(wi.v, MR.one, 32);
    for (size_t i = 0; i < n; i++) {
        memset(&acc, 0, sizeof acc);
        memcpy(wij.v, MR.one, 32);
        for (size_t j = 0; j < n; j++) {
            mmul_(&MR, t.v, in + 4 * j, wij.v);
            madd_(&MR, acc.v, acc.v, t.v);
            mmul_(&MR, wij.v, wij.v, wi.v);
        }
        memcpy(buf + 4 * i, acc.v, 32);
        mmul_(&MR, wi.v, wi.v, w.v);
    }
    if (inverse) {
        orc_fe sc;
        memcpy(sc.v, MR.one, 32);
        for (int i = 0; i < log_n; i++) mmul_(&MR, sc.v, sc.v, FR_HALF.v);
        for (size_t i = 0; i < n; i++) mmul_(&MR, buf + 4 * i, buf + 4 * i, sc.v);
    }
    memcpy(out, buf, n * 32);
    free(buf);
}

void orc_coset_ntt_mt(uint64_t* out, const uint64_t* in, int log_n, int inverse, const orc_fe* g, int nthreads) {
    INIT();
    size_t n = (size_t)1 << log_n;
    orc_fe gp, gs = *g;
    memcpy(gp.v, MR.one, 32);
    if (!inverse) {
        uint64_t* tmp = (uint64_t*)malloc(n * 32);
        for (size_t i = 0; i < n; i++) {
            mmul_(&MR, tmp + 4 * i, in + 4 * i, gp.v);
            mmul_(&MR, gp.v, gp.v, gs.v);
        }
        orc_ntt_mt(out, tmp, log_n, 0, nthreads);
        free(tmp);
    } else {
        orc_fe gi;
        minv_(&MR, gi.v, gs.v);
        orc_ntt_mt(out, in, log_n, 1, nthreads);
        for (size_t i = 0; i < n; i++) {
            mmul_(&MR, out + 4 * i, out + 4 * i, gp.v);
            mmul_(&MR, gp.v, gp.v, gi.v);
        }
    }
}

void orc_coset_ntt(uint64_t* out, const uint64_t* in, int log_n, int inverse, const orc_fe* g) {
    orc_coset_ntt_mt(out, in, log_n, inverse, g, 1);
}

/* compute_h after the sparse matvec (groth16.cu:322-383): 3 INTT, coset shift
 * g = 5 (7 if 5^n = 1), 3 forward NTT, pointwise (A*B - C) / (g^n - 1),
 * INTT, unscale by g^-i. */
void orc_compute_h_from_evals(uint64_t* h, const uint64_t* a_eval, const uint64_t* b_eval,
                              const uint64_t* c_eval, int log_n) {
    INIT();
    size_t n = (size_t)1 << log_n;
    uint64_t* A = (uint64_t*)malloc(n * 32);
    uint64_t* B = (uint64_t*)malloc(n * 32);
    uint64_t* C = (uint64_t*)malloc(n * 32);
    orc_ntt(A, a_eval, log_n, 1);
    orc_ntt(B, b_eval, log_n, 1);
    orc_ntt(C, c_eval, log_n, 1);
    orc_fe g, z;
    orc_fr_from_u64(&g, 5);
    z = g;
    for (int i = 0; i < log_n; i++) mmul_(&MR, z.v, z.v, z.v);
    msub_(&MR, z.v, z.v, MR.one);
    if (fe_is_zero(&z)) {
        orc_fr_from_u64(&g, 7);
        z = g;
        for (int i = 0; i < log_n; i++) mmul_(&MR, z.v, z.v, z.v);
        msub_(&MR, z.v, z.v, MR.one);
    }
    orc_coset_ntt(A, A, log_n, 0, &g);
    orc_coset_ntt(B, B, log_n, 0, &g);
    orc_coset_ntt(C, C, log_n, 0, &g);
    orc_fe zi;
    minv_(&MR, zi.v, z.v);
    for (size_t j = 0; j < n; j++) {
        uint64_t t[4];
        mmul_(&MR, t, A + 4 * j, B + 4 * j);
        msub_(&MR, t, t, C + 4 * j);
        mmul_(&MR, A + 4 * j, t, zi.v);
    }
    orc_coset_ntt(h, A, log_n, 1, &g);
    free(A); free(B); free(C);
}

/* ------------------------------------------------------------------ */
/* mt19937_64 (Matsumoto & Nishimura 2000; the std::mt19937_64 engine)   */
/* ------------------------------------------------------------------ */
void orc_rng_seed(orc_rng* r, uint64_t seed) {
    r->mt[0] = seed;
    for (int i = 1; i < 312; i++)
        r->mt[i] = 6364136223846793005ULL * (r->mt[i - 1] ^ (r->mt[i - 1] >> 62)) + (uint64_t)i;
    r->idx = 312;
}
uint64_t orc_rng_next(orc_rng* r) {
    static const uint64_t UM = 0xFFFFFFFF80000000ULL, LM = 0x7FFFFFFFULL;
    if (r->idx >= 312) {
        for (int i = 0; i < 312; i++) {
            uint64_t x = (r->mt[i] & UM) | (r->mt[(i + 1) % 312] & LM);
            uint64_t xa = x >> 1;
            if (x & 1) xa ^= 0xB5026F5AA96619E9ULL;
            r->mt[i] = r->mt[(i + 156) % 312] ^ xa;
        }
        r->idx = 0;
    }
    uint64_t x = r->mt[r->idx++];
    x ^= (x >> 29) & 0x5555555555555555ULL;
    x ^= (x << 17) & 0x71D67FFFEDA60000ULL;
    x ^= (x << 37) & 0xFFF7EEE000000000ULL;
    x ^= (x >> 43);
    return x;
}
void orc_rand_fr(orc_rng* r, orc_fe* out) {
    INIT();
    uint64_t s[4];
    do {
        for (int i = 0; i < 4; i++) s[i] = orc_rng_next(r);
        s[3] &= (1ULL << 62) - 1;
    } while (geq(s, MR.m));
    mmul_(&MR, out->v, s, MR.r2);
}

void orc_rand_fr_vec(orc_rng* r, uint64_t* out, size_t n) {
    for (size_t i = 0; i < n; i++) orc_rand_fr(r, (orc_fe*)(out + 4 * i));
}

int orc_g2_is_on_curve_raw(const uint64_t* p128) {
    orc_g2a a;
    g2_load(&a, p128);
    return orc_g2_is_on_curve(&a);
}

/* ------------------------------------------------------------------ */
/* fixed-base generators for synthetic inputs                           */
/* ------------------------------------------------------------------ */
/* G1 comb: T[j][d] = d * 2^(8j) * G (affine), k*G = sum_j T[j][byte_j(k)] */
static orc_g1a* g_g1_comb;
static pthread_once_t g_comb_once = PTHREAD_ONCE_INIT;

static void g1_comb_init(void) {
    INIT();
    g_g1_comb = (orc_g1a*)malloc(32 * 256 * sizeof(orc_g1a));
    orc_g1a g;
    orc_g1_generator(&g);
    orc_g1j base, acc;
    orc_g1_from_affine(&base, &g);
    for (int j = 0; j < 32; j++) {
        orc_g1_identity(&acc);
        memset(&g_g1_comb[j * 256], 0, sizeof(orc_g1a));
        g_g1_comb[j * 256].inf = 1;
        for (int d = 1; d < 256; d++) {
            orc_g1_add(&acc, &acc, &base);
            orc_g1_to_affine(&g_g1_comb[j * 256 + d], &acc);
        }
        for (int i = 0; i < 8; i++) orc_g1_dbl(&base, &base);
    }
}

typedef struct { uint64_t* out; const uint64_t* sc; size_t i0, i1; } fb_job;

static void* g1_fb_worker(void* arg) {
    fb_job* J = (fb_job*)arg;
    for (size_t i = J->i0; i < J->i1; i++) {
        uint64_t s[4];
        orc_fr_to_std(s, (const orc_fe*)(J->sc + 4 * i));
        orc_g1j acc;
        orc_g1_identity(&acc);
        for (int j = 0; j < 32; j++) {
            int d = (int)((s[j >> 3] >> (8 * (j & 7))) & 0xFF);
            if (d) orc_g1_madd(&acc, &acc, &g_g1_comb[j * 256 + d]);
        }
        orc_g1a a;
        orc_g1_to_affine(&a, &acc);
        if (a.inf) memset(J->out + 8 * i, 0, 64);
        else { memcpy(J->out + 8 * i, a.x.v, 32); memcpy(J->out + 8 * i + 4, a.y.v, 32); }
    }
    return NULL;
}

static void run_parallel(void* (*fn)(void*), uint64_t* out, const uint64_t* sc, size_t n, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if ((size_t)nthreads > n) nthreads = n ? (int)n : 1;
    pthread_t* th = (pthread_t*)malloc(nthreads * sizeof(pthread_t));
    fb_job* jobs = (fb_job*)malloc(nthreads * sizeof(fb_job));
    for (int t = 0; t < nthreads; t++) {
        jobs[t].out = out; jobs[t].sc = sc;
        jobs[t].i0 = n * t / nthreads; jobs[t].i1 = n * (t + 1) / nthreads;
        pthread_create(&th[t], NULL, fn, &jobs[t]);
    }
    for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
    free(th); free(jobs);
}

void orc_g1_fixed_base(uint64_t* out64, const uint64_t* scalars, size_t n, int nthreads) {
    pthread_once(&g_comb_once, g1_comb_init);
    run_parallel(g1_fb_worker, out64, scalars, n, nthreads);
}

/* G2 Jacobian formulas over Fp2 (a = 0): dbl-2009-l and add-2007-bl
 * (Explicit-Formulas Database), used only to generate test points. */
static void g2j_dbl(orc_g2j* r, const orc_g2j* p) {
    if (f2_is_zero(&p->z)) { *r = *p; return; }
    orc_fe2 A, B, C, D, E, F, t, X3, Y3, Z3, C8;
    f2_sqr(&A, &p->x); f2_sqr(&B, &p->y); f2_sqr(&C, &B);
    f2_add(&t, &p->x, &B); f2_sqr(&D, &t); f2_sub(&D, &D, &A); f2_sub(&D, &D, &C); f2_add(&D, &D, &D);
    f2_add(&E, &A, &A); f2_add(&E, &E, &A);
    f2_sqr(&F, &E);
    f2_sub(&X3, &F, &D); f2_sub(&X3, &X3, &D);
    f2_add(&C8, &C, &C); f2_add(&C8, &C8, &C8); f2_add(&C8, &C8, &C8);
    f2_sub(&t, &D, &X3); f2_mul(&Y3, &E, &t); f2_sub(&Y3, &Y3, &C8);
    f2_mul(&Z3, &p->y, &p->z); f2_add(&Z3, &Z3, &Z3);
    r->x = X3; r->y = Y3; r->z = Z3;
}
static void g2j_add(orc_g2j* r, const orc_g2j* p, const orc_g2j* q) {
    if (f2_is_zero(&p->z)) { *r = *q; return; }
    if (f2_is_zero(&q->z)) { *r = *p; return; }
    orc_fe2 Z1Z1, Z2Z2, U1, U2, S1, S2, H, Rr, HH, HHH, V, X3, Y3, Z3, t;
    f2_sqr(&Z1Z1, &p->z); f2_sqr(&Z2Z2, &q->z);
    f2_mul(&U1, &p->x, &Z2Z2); f2_mul(&U2, &q->x, &Z1Z1);
    f2_mul(&t, &p->y, &q->z); f2_mul(&S1, &t, &Z2Z2);
    f2_mul(&t, &q->y, &p->z); f2_mul(&S2, &t, &Z1Z1);
    f2_sub(&H, &U2, &U1); f2_sub(&Rr, &S2, &S1);
    if (f2_is_zero(&H)) {
        if (f2_is_zero(&Rr)) { g2j_dbl(r, p); return; }
        orc_g2_identity(r); return;
    }
    f2_sqr(&HH, &H); f2_mul(&HHH, &HH, &H); f2_mul(&V, &U1, &HH);
    f2_sqr(&X3, &Rr); f2_sub(&X3, &X3, &HHH); f2_sub(&X3, &X3, &V); f2_sub(&X3, &X3, &V);
    f2_sub(&t, &V, &X3); f2_mul(&Y3, &Rr, &t); f2_mul(&t, &S1, &HHH); f2_sub(&Y3, &Y3, &t);
    f2_mul(&t, &p->z, &q->z); f2_mul(&Z3, &t, &H);
    r->x = X3; r->y = Y3; r->z = Z3;
}

static orc_g2j* g_g2_comb;
static pthread_once_t g_comb2_once = PTHREAD_ONCE_INIT;
static void g2_comb_init(void) {
    INIT();
    g_g2_comb = (orc_g2j*)malloc(32 * 256 * sizeof(orc_g2j));
    orc_g2j base, acc;
    orc_g2_from_affine(&base, &G2_GEN);
    for (int j = 0; j < 32; j++) {
        orc_g2_identity(&acc);
        g_g2_comb[j * 256] = acc;
        for (int d = 1; d < 256; d++) {
            g2j_add(&acc, &acc, &base);
            g_g2_comb[j * 256 + d] = acc;
        }
        for (int i = 0; i < 8; i++) g2j_dbl(&base, &base);
    }
}
static void* g2_fb_worker(void* arg) {
    fb_job* J = (fb_job*)arg;
    for (size_t i = J->i0; i < J->i1; i++) {
        uint64_t s[4];
        orc_fr_to_std(s, (const orc_fe*)(J->sc + 4 * i));
        orc_g2j acc;
        orc_g2_identity(&acc);
        for (int j = 0; j < 32; j++) {
            int d = (int)((s[j >> 3] >> (8 * (j & 7))) & 0xFF);
            if (d) g2j_add(&acc, &acc, &g_g2_comb[j * 256 + d]);
        }
        orc_g2a a;
        orc_g2_to_affine(&a, &acc);
        uint64_t* o = J->out + 16 * i;
        if (a.inf) memset(o, 0, 128);
        else { memcpy(o, a.x.c0.v, 32); memcpy(o + 4, a.x.c1.v, 32); memcpy(o + 8, a.y.c0.v, 32); memcpy(o + 12, a.y.c1.v, 32); }
    }
    return NULL;
}
void orc_g2_fixed_base(uint64_t* out128, const uint64_t* scalars, size_t n, int nthreads) {
    pthread_once(&g_comb2_once, g2_comb_init);
    run_parallel(g2_fb_worker, out128, scalars, n, nthreads);
}

/* ------------------------------------------------------------------ */
/* full-size property helpers                                           */
/* ------------------------------------------------------------------ */
typedef struct { const uint64_t *a, *b; size_t i0, i1; orc_fe acc; } dot_job;
static void* dot_worker(void* arg) {
    dot_job* J = (dot_job*)arg;
    memset(&J->acc, 0, sizeof J->acc);
    for (size_t i = J->i0; i < J->i1; i++) {
        uint64_t t[4];
        mmul_(&MR, t, J->a + 4 * i, J->b + 4 * i);
        madd_(&MR, J->acc.v, J->acc.v, t);
    }
    return NULL;
}
void orc_fr_dot(orc_fe* out, const uint64_t* a, const uint64_t* b, size_t n, int nthreads) {
    INIT();
    if (nthreads < 1) nthreads = 1;
    pthread_t* th = (pthread_t*)malloc(nthreads * sizeof(pthread_t));
    dot_job* jobs = (dot_job*)malloc(nthreads * sizeof(dot_job));
    for (int t = 0; t < nthreads; t++) {
        jobs[t].a = a; jobs[t].b = b; jobs[t].i0 = n * t / nthreads; jobs[t].i1 = n * (t + 1) / nthreads;
        pthread_create(&th[t], NULL, dot_worker, &jobs[t]);
    }
    memset(out, 0, sizeof *out);
    for (int t = 0; t < nthreads; t++) {
        pthread_join(th[t], NULL);
        madd_(&MR, out->v, out->v, jobs[t].acc.v);
    }
    free(th); free(jobs);
}
void orc_fr_poly_eval(orc_fe* out, const uint64_t* coeffs, size_t n, const orc_fe* x) {
    INIT();
    orc_fe acc;
    memset(&acc, 0, sizeof acc);
    for (size_t i = n; i-- > 0;) {
        mmul_(&MR, acc.v, acc.v, x->v);
        madd_(&MR, acc.v, acc.v, coeffs + 4 * i);
    }
    *out = acc;
}
