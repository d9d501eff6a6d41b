// pairing.cpp -- the BN254 optimal ate pairing and the Groth16 verifier
// (Groth16Verifier::verify, src/prover/groth16.cu:967-1022, over
// verify_pairing_product, src/curve/pairing.cuh:198-282), host code with the
// public-input sum vk_x = IC[0] + sum_i x_i IC[i+1] as an MSM on the GPU.
//
// Tower (the reference's, src/field/fp6.cuh, fp12.cuh): Fp2 = Fp[u]/(u^2 + 1),
// Fp6 = Fp2[v]/(v^3 - xi) with xi = 9 + u, Fp12 = Fp6[w]/(w^2 - v).  G2 is the
// D-type sextic twist E': y^2 = x^3 + 3/xi, untwisted by (x, y) -> (x w^2, y w^3).
//
// Miller loop (the optimal ate pairing of Vercauteren, "Optimal pairings",
// 2010, for BN curves): f_{6t+2, Q}(P) over the signed binary expansion of
// 6t + 2 (t = 4965661367192848881, the BN parameter), then the lines through
// [6t+2]Q and pi(Q), and through that sum and -pi^2(Q), pi the p-power
// Frobenius.  Points of the loop are projective (no inversion in the loop);
// the line through T with slope l (on the twist), evaluated at P = (xP, yP), is,
// up to a factor in Fp2,
//   yP - l xP w + (l xT - yT) w^3,
// vertical lines omitted (they lie in a proper subfield and vanish under the
// final exponentiation).
//
// Final exponentiation f^((p^12 - 1)/r) = f^((p^6 - 1)(p^2 + 1) d) with the
// hard part d = (p^4 - p^2 + 1)/r written in base p (Scott, Benger, Charlemagne,
// Dominguez Perez, Kachisa, "On the final exponentiation for calculating
// pairings on ordinary elliptic curves", 2009):
//   d = l0 + l1 p + l2 p^2 + p^3,  l2 = 6t^2 + 1,
//   l1 = -36t^3 - 18t^2 - 12t + 1,  l0 = -36t^3 - 30t^2 - 18t - 2,
// checked at start-up against d r = p^4 - p^2 + 1.  The result is exactly the
// reduced pairing value (the reference raises to the same exponent in one
// chain), so pairing values compare bit for bit.  Every constant (the Frobenius
// coefficients xi^(i (p - 1)/6), the loop digits, the l_i) is derived here
// from p, xi and t.
#include "host_field.hpp"
#include "runtime.cuh"

#include <cstring>
#include <mutex>
#include <vector>

namespace zkp {

using zkh::Fe;
using zkh::Fp2;

// ---------------------------------------------------------------- Fp2 extras
static Fp2 f2(const Fe& a, const Fe& b) { Fp2 r; r.c0 = a; r.c1 = b; return r; }
static Fp2 add(const Fp2& a, const Fp2& b) { Fp2 r; zkh::fadd(r, a, b); return r; }
static Fp2 sub(const Fp2& a, const Fp2& b) { Fp2 r; zkh::fsub(r, a, b); return r; }
static Fp2 mul(const Fp2& a, const Fp2& b) { Fp2 r; zkh::fmul(r, a, b); return r; }
// (a0 + a1 u)^2 = (a0 + a1)(a0 - a1) + 2 a0 a1 u: two products
static Fp2 sqr(const Fp2& a) {
    Fe s, d, t;
    zkh::fadd(s, a.c0, a.c1);
    zkh::fsub(d, a.c0, a.c1);
    Fp2 r;
    zkh::fmul(r.c0, s, d);
    zkh::fmul(t, a.c0, a.c1);
    zkh::fadd(r.c1, t, t);
    return r;
}
static Fp2 neg(const Fp2& a) { Fp2 z; zkh::fset_zero(z); return sub(z, a); }
static Fp2 inv(const Fp2& a) { Fp2 r; zkh::finv(r, a); return r; }
static Fp2 conj(const Fp2& a) { Fp2 r; r.c0 = a.c0; zkh::fsub(r.c1, zkh::zero(), a.c1); return r; }
static Fp2 mul_fp(const Fp2& a, const Fe& s) { Fp2 r; zkh::fmul(r.c0, a.c0, s); zkh::fmul(r.c1, a.c1, s); return r; }
static Fp2 one2() { Fp2 r; zkh::fset_one(r); return r; }
static Fp2 zero2() { Fp2 r; zkh::fset_zero(r); return r; }
static bool eq(const Fp2& a, const Fp2& b) { return zkh::eq(a.c0, b.c0) && zkh::eq(a.c1, b.c1); }
static Fe fp_small(uint64_t v) {
    uint64_t s[4] = {v, 0, 0, 0};
    Fe r;
    zkh::from_std(zkh::kP, r, s);
    return r;
}
// xi = 9 + u; (a0 + a1 u)(9 + u) = (9 a0 - a1) + (a0 + 9 a1) u, by additions
static Fp2 xi() { return f2(fp_small(9), fp_small(1)); }
static Fe times9(const Fe& a) {
    Fe t;
    zkh::fadd(t, a, a);  // 2a
    zkh::fadd(t, t, t);  // 4a
    zkh::fadd(t, t, t);  // 8a
    zkh::fadd(t, t, a);  // 9a
    return t;
}
static Fp2 mul_xi(const Fp2& a) {
    Fp2 r;
    zkh::fsub(r.c0, times9(a.c0), a.c1);
    zkh::fadd(r.c1, a.c0, times9(a.c1));
    return r;
}
static Fp2 pow2(const Fp2& a, const uint64_t e[4]) {
    Fp2 acc = one2();
    for (int bit = 255; bit >= 0; bit--) {
        acc = sqr(acc);
        if ((e[bit >> 6] >> (bit & 63)) & 1) acc = mul(acc, a);
    }
    return acc;
}

// ---------------------------------------------------------------- Fp6, Fp12
struct Fp6 {
    Fp2 c0, c1, c2;
};
static Fp6 add(const Fp6& a, const Fp6& b) { return {add(a.c0, b.c0), add(a.c1, b.c1), add(a.c2, b.c2)}; }
static Fp6 sub(const Fp6& a, const Fp6& b) { return {sub(a.c0, b.c0), sub(a.c1, b.c1), sub(a.c2, b.c2)}; }
static Fp6 neg(const Fp6& a) { return {neg(a.c0), neg(a.c1), neg(a.c2)}; }
static Fp6 mul(const Fp6& a, const Fp6& b) {
    // v^3 = xi; Karatsuba: six Fp2 products
    const Fp2 t0 = mul(a.c0, b.c0), t1 = mul(a.c1, b.c1), t2 = mul(a.c2, b.c2);
    const Fp2 s12 = sub(sub(mul(add(a.c1, a.c2), add(b.c1, b.c2)), t1), t2);  // a1 b2 + a2 b1
    const Fp2 s01 = sub(sub(mul(add(a.c0, a.c1), add(b.c0, b.c1)), t0), t1);  // a0 b1 + a1 b0
    const Fp2 s02 = sub(sub(mul(add(a.c0, a.c2), add(b.c0, b.c2)), t0), t2);  // a0 b2 + a2 b0
    return {add(t0, mul_xi(s12)), add(s01, mul_xi(t2)), add(s02, t1)};
}
static Fp6 mul_v(const Fp6& a) { return {mul_xi(a.c2), a.c0, a.c1}; }
static Fp6 one6() { return {one2(), zero2(), zero2()}; }
static Fp6 inv(const Fp6& a) {
    const Fp2 A = sub(sqr(a.c0), mul_xi(mul(a.c1, a.c2)));
    const Fp2 B = sub(mul_xi(sqr(a.c2)), mul(a.c0, a.c1));
    const Fp2 C = sub(sqr(a.c1), mul(a.c0, a.c2));
    const Fp2 F = add(mul(a.c0, A), mul_xi(add(mul(a.c2, B), mul(a.c1, C))));
    const Fp2 Fi = inv(F);
    return {mul(A, Fi), mul(B, Fi), mul(C, Fi)};
}

struct Fp12 {
    Fp6 c0, c1;
};
static Fp12 mul(const Fp12& a, const Fp12& b) {  // w^2 = v; Karatsuba: three Fp6 products
    const Fp6 t0 = mul(a.c0, b.c0), t1 = mul(a.c1, b.c1);
    const Fp6 s = sub(sub(mul(add(a.c0, a.c1), add(b.c0, b.c1)), t0), t1);
    return {add(t0, mul_v(t1)), s};
}
// (a0 + a1 w)^2 = (a0 + a1)(a0 + v a1) - t - v t + 2 t w, t = a0 a1: two Fp6 products
static Fp12 sqr(const Fp12& a) {
    const Fp6 t = mul(a.c0, a.c1);
    const Fp6 c0 = sub(sub(mul(add(a.c0, a.c1), add(a.c0, mul_v(a.c1))), t), mul_v(t));
    return {c0, add(t, t)};
}
static Fp12 conj(const Fp12& a) { return {a.c0, neg(a.c1)}; }
static Fp12 one12() { return {one6(), {zero2(), zero2(), zero2()}}; }
static Fp12 inv(const Fp12& a) {  // (c0 - c1 w) / (c0^2 - v c1^2)
    const Fp6 d = inv(sub(mul(a.c0, a.c0), mul_v(mul(a.c1, a.c1))));
    return {mul(a.c0, d), neg(mul(a.c1, d))};
}
static bool eq(const Fp12& a, const Fp12& b) {
    const Fp2* x = &a.c0.c0;
    const Fp2* y = &b.c0.c0;
    for (int i = 0; i < 6; i++)
        if (!eq(x[i], y[i])) return false;
    return true;
}

// ---------------------------------------------------------------- derived constants
struct Consts {
    Fp2 gamma[6];          // xi^(i (p - 1)/6): (w^i)^p = w^i gamma[i]
    Fp2 b3;                // 3 b' = 9 / xi, b' = 3 / xi the twist's constant
    std::vector<int> naf;  // signed digits of 6t + 2, least significant first
    uint64_t l0[4], l1[4], l2[4];  // |l0|, |l1|, l2 (l0, l1 < 0)
    bool ok = false;
};

// little helpers on multi-limb unsigned integers (up to 17 limbs)
static void mul_small(uint64_t* r, const uint64_t* a, int n, uint64_t k) {
    unsigned __int128 c = 0;
    for (int i = 0; i < n; i++) {
        c += (unsigned __int128)a[i] * k;
        r[i] = (uint64_t)c;
        c >>= 64;
    }
}
static void add_n(uint64_t* r, const uint64_t* a, const uint64_t* b, int n) {
    unsigned __int128 c = 0;
    for (int i = 0; i < n; i++) {
        c += (unsigned __int128)a[i] + b[i];
        r[i] = (uint64_t)c;
        c >>= 64;
    }
}
static void sub_n(uint64_t* r, const uint64_t* a, const uint64_t* b, int n) {
    uint64_t br = 0;
    for (int i = 0; i < n; i++) {
        unsigned __int128 d = (unsigned __int128)a[i] - b[i] - br;
        r[i] = (uint64_t)d;
        br = (uint64_t)(d >> 64) & 1;
    }
}
static void mul_n(uint64_t* r, const uint64_t* a, int na, const uint64_t* b, int nb) {  // r: na + nb limbs
    std::memset(r, 0, (size_t)(na + nb) * 8);
    for (int i = 0; i < na; i++) {
        unsigned __int128 c = 0;
        for (int j = 0; j < nb; j++) {
            c += (unsigned __int128)a[i] * b[j] + r[i + j];
            r[i + j] = (uint64_t)c;
            c >>= 64;
        }
        r[i + nb] = (uint64_t)c;
    }
}

static const uint64_t kT = 4965661367192848881ull;  // the BN parameter of BN254

static Consts make_consts() {
    Consts C;
    // gamma[i] = xi^(i (p - 1)/6)
    uint64_t e[4];
    std::memcpy(e, zkh::kP.m, 32);
    e[0] -= 1;  // p - 1 (p odd)
    // divide by 6
    unsigned __int128 rem = 0;
    for (int i = 3; i >= 0; i--) {
        unsigned __int128 cur = (rem << 64) | e[i];
        e[i] = (uint64_t)(cur / 6);
        rem = cur % 6;
    }
    if (rem != 0) return C;
    const Fp2 g1 = pow2(xi(), e);
    C.gamma[0] = one2();
    for (int i = 1; i < 6; i++) C.gamma[i] = mul(C.gamma[i - 1], g1);
    C.b3 = mul(f2(fp_small(9), zkh::zero()), inv(xi()));
    // NAF of 6t + 2
    {
        uint64_t s[2];
        unsigned __int128 v = (unsigned __int128)kT * 6 + 2;
        s[0] = (uint64_t)v;
        s[1] = (uint64_t)(v >> 64);
        unsigned __int128 k = ((unsigned __int128)s[1] << 64) | s[0];
        while (k) {
            int d = 0;
            if (k & 1) {
                d = 2 - (int)(k & 3);  // 1 or -1
                if (d == 1) k -= 1; else k += 1;
            }
            C.naf.push_back(d);
            k >>= 1;
        }
    }
    // l2 = 6t^2 + 1, |l1| = 36t^3 + 18t^2 + 12t - 1, |l0| = 36t^3 + 30t^2 + 18t + 2
    uint64_t t[4] = {kT, 0, 0, 0}, t2[8], t3[8], a[4], b[4];
    mul_n(t2, t, 1, t, 1);  // 2 limbs
    mul_n(t3, t2, 2, t, 1); // 3 limbs
    for (int i = 2; i < 4; i++) t2[i] = 0;
    t3[3] = 0;
    uint64_t one[4] = {1, 0, 0, 0}, two[4] = {2, 0, 0, 0};
    mul_small(C.l2, t2, 4, 6);
    add_n(C.l2, C.l2, one, 4);
    mul_small(a, t3, 4, 36);
    mul_small(b, t2, 4, 18);
    add_n(a, a, b, 4);
    mul_small(b, t, 4, 12);
    add_n(a, a, b, 4);
    sub_n(C.l1, a, one, 4);
    mul_small(a, t3, 4, 36);
    mul_small(b, t2, 4, 30);
    add_n(a, a, b, 4);
    mul_small(b, t, 4, 18);
    add_n(a, a, b, 4);
    add_n(C.l0, a, two, 4);
    // check d r = p^4 - p^2 + 1 with d = p^3 + l2 p^2 - |l1| p - |l0| (p^4 < 2^1016: 17 limbs)
    const int W = 17;
    uint64_t p1[W] = {}, p2[W] = {}, p3[W] = {}, p4[W] = {}, tmp[2 * W];
    std::memcpy(p1, zkh::kP.m, 32);
    mul_n(tmp, p1, 4, p1, 4);
    std::memcpy(p2, tmp, 8 * 8);
    mul_n(tmp, p2, 8, p1, 4);
    std::memcpy(p3, tmp, 12 * 8);
    mul_n(tmp, p2, 8, p2, 8);
    std::memcpy(p4, tmp, 16 * 8);
    uint64_t d[W] = {}, u[W] = {};
    std::memcpy(d, p3, sizeof d);
    mul_n(tmp, p2, 8, C.l2, 4);
    std::memcpy(u, tmp, 12 * 8);
    add_n(d, d, u, W);
    mul_n(tmp, p1, 4, C.l1, 4);
    std::memset(u, 0, sizeof u);
    std::memcpy(u, tmp, 8 * 8);
    sub_n(d, d, u, W);
    std::memset(u, 0, sizeof u);
    std::memcpy(u, C.l0, 32);
    sub_n(d, d, u, W);
    uint64_t r[W] = {}, lhs[2 * W], rhs[W];
    std::memcpy(r, zkh::kR.m, 32);
    mul_n(lhs, d, W, r, 4);  // d r (fits in 13 limbs)
    std::memcpy(rhs, p4, sizeof rhs);
    sub_n(rhs, rhs, p2, W);
    uint64_t o[W] = {1};
    add_n(rhs, rhs, o, W);
    C.ok = std::memcmp(lhs, rhs, sizeof rhs) == 0;
    for (int i = W; i < W + 4; i++) C.ok = C.ok && lhs[i] == 0;
    return C;
}

static const Consts& consts() {
    static std::once_flag once;
    static Consts C;
    std::call_once(once, [] { C = make_consts(); });
    return C;
}

// ---------------------------------------------------------------- Frobenius, exponentiation
static Fp12 frob(const Fp12& a) {
    const Consts& C = consts();
    // coefficient of w^i: i = 0, 2, 4 in c0 (c0, c1, c2), i = 1, 3, 5 in c1
    Fp12 r;
    r.c0.c0 = mul(conj(a.c0.c0), C.gamma[0]);
    r.c0.c1 = mul(conj(a.c0.c1), C.gamma[2]);
    r.c0.c2 = mul(conj(a.c0.c2), C.gamma[4]);
    r.c1.c0 = mul(conj(a.c1.c0), C.gamma[1]);
    r.c1.c1 = mul(conj(a.c1.c1), C.gamma[3]);
    r.c1.c2 = mul(conj(a.c1.c2), C.gamma[5]);
    return r;
}
// Squaring in the cyclotomic subgroup (order p^4 - p^2 + 1), after Granger and
// Scott, "Faster squaring in the cyclotomic subgroup of sixth degree
// extensions" (PKC 2010).  With X = w and Y = w^3 (Y^2 = xi, X^3 = Y) an element
// is a0 + a1 X + a2 X^2 over Fp4 = Fp2[Y], with a0 = c0.c0 + c1.c1 Y,
// a1 = c1.c0 + c0.c2 Y, a2 = c0.c1 + c1.c2 Y, and its square is
//   (3 a0^2 - 2 conj(a0)) + (3 Y a2^2 + 2 conj(a1)) X + (3 a1^2 - 2 conj(a2)) X^2,
// conj: Y -> -Y.  Three Fp4 squarings (x + y Y)^2 = (x^2 + xi y^2) + 2 x y Y.
static void fp4_sqr(Fp2& r0, Fp2& r1, const Fp2& x, const Fp2& y) {
    const Fp2 xy = mul(x, y);
    r0 = add(sqr(x), mul_xi(sqr(y)));
    r1 = add(xy, xy);
}
static Fp2 times3(const Fp2& a) { return add(add(a, a), a); }
static Fp2 twice(const Fp2& a) { return add(a, a); }
static Fp12 cyclotomic_sqr(const Fp12& a) {
    Fp2 s0, s1, t0, t1, u0, u1;
    fp4_sqr(s0, s1, a.c0.c0, a.c1.c1);  // a0^2
    fp4_sqr(t0, t1, a.c1.c0, a.c0.c2);  // a1^2
    fp4_sqr(u0, u1, a.c0.c1, a.c1.c2);  // a2^2
    Fp12 r;
    r.c0.c0 = sub(times3(s0), twice(a.c0.c0));        // 3 Re(a0^2) - 2 Re(a0)
    r.c1.c1 = add(times3(s1), twice(a.c1.c1));        // 3 Im(a0^2) + 2 Im(a0)
    r.c1.c0 = add(times3(mul_xi(u1)), twice(a.c1.c0));  // Y a2^2 = xi Im + Re Y
    r.c0.c2 = sub(times3(u0), twice(a.c0.c2));
    r.c0.c1 = sub(times3(t0), twice(a.c0.c1));
    r.c1.c2 = add(times3(t1), twice(a.c1.c2));
    return r;
}
// a^e for a in the cyclotomic subgroup
static Fp12 pow_cyclotomic(const Fp12& a, const uint64_t e[4]) {
    Fp12 acc = one12();
    int top = 255;
    while (top >= 0 && !((e[top >> 6] >> (top & 63)) & 1)) top--;
    for (int bit = top; bit >= 0; bit--) {
        acc = cyclotomic_sqr(acc);
        if ((e[bit >> 6] >> (bit & 63)) & 1) acc = mul(acc, a);
    }
    return acc;
}
// The hard part m^d, d = l0 + l1 p + l2 p^2 + p^3, from A = m^t, B = m^(t^2),
// Cc = m^(t^3) (three exponentiations by the 63-bit t) and short chains for the
// small coefficients: m^l2 = B^6 m, m^l1 = conj(Cc^36 B^18 A^12) m,
// m^l0 = conj(Cc^36 B^30 A^18 m^2) (conj inverts in the cyclotomic subgroup).
// The same exponent as one exponentiation by each l_i, in about a third of the
// operations.
static Fp12 final_exp(const Fp12& f) {
    Fp12 m = mul(conj(f), inv(f));  // f^(p^6 - 1)
    m = mul(frob(frob(m)), m);       // ^(p^2 + 1): now in the cyclotomic subgroup
    const uint64_t te[4] = {kT, 0, 0, 0};
    const Fp12 A = pow_cyclotomic(m, te), B = pow_cyclotomic(A, te), Cc = pow_cyclotomic(B, te);
    auto sq = [](const Fp12& x) { return cyclotomic_sqr(x); };
    const Fp12 A2 = sq(A), A4 = sq(A2), A8 = sq(A4), A16 = sq(A8);
    const Fp12 B2 = sq(B), B4 = sq(B2), B8 = sq(B4), B16 = sq(B8);
    const Fp12 C4 = sq(sq(Cc)), C32 = sq(sq(sq(C4)));
    const Fp12 C36 = mul(C32, C4);
    const Fp12 m_l2 = mul(mul(B4, B2), m);                                         // B^6 m
    const Fp12 m_l1 = mul(conj(mul(mul(C36, mul(B16, B2)), mul(A8, A4))), m);     // conj(Cc^36 B^18 A^12) m
    const Fp12 m_l0 = conj(mul(mul(C36, mul(mul(B16, B8), mul(B4, B2))), mul(mul(A16, A2), sq(m))));
    return mul(mul(m_l0, frob(m_l1)), mul(frob(frob(m_l2)), frob(frob(frob(m)))));
}

// ---------------------------------------------------------------- Miller loop
struct G1a {
    Fe x, y;
    bool inf;
};
struct G2a {
    Fp2 x, y;
    bool inf;
};

// Points of the loop in homogeneous projective coordinates on the twist,
// (X : Y : Z) for (X / Z, Y / Z), so that no step inverts.  A line is the
// affine line yP - l xP w + (l xT - yT) w^3 times a factor in Fp2, which the
// final exponentiation removes (Costello, Lange and Naehrig, "Faster pairing
// computations on curves with high-degree twists", PKC 2010; the point formulas
// after Aranha, Karabina, Longa, Gebotys and Lopez, Eurocrypt 2011).
struct G2p {
    Fp2 x, y, z;
};
static Fp12 line3(const Fp2& c_y, const Fp2& c_x, const Fp2& c_w3, const G1a& P) {
    // c_y yP + c_x xP w + c_w3 w^3
    Fp12 r = {{mul_fp(c_y, P.y), zero2(), zero2()}, {mul_fp(c_x, P.x), c_w3, zero2()}};
    return r;
}
// T <- 2T; the tangent at T times 2 Y Z^2 / Z = 2 Y Z:
//   2 Y Z yP - 3 X^2 xP w + (Y^2 - 3 b' Z^2) w^3
// (from 3 X^3 - 2 Y^2 Z = Z (Y^2 - 3 b' Z^2) on Y^2 Z = X^3 + b' Z^3).  The new
// point is the standard doubling scaled by 4 to avoid halving:
//   (2 X Y (Y^2 - 9 b' Z^2), (Y^2 + 9 b' Z^2)^2 - 12 (3 b' Z^2)^2, 8 Y^3 Z)
static Fp12 dbl_step(G2p& T, const G1a& P) {
    const Consts& C = consts();
    const Fp2 B = sqr(T.y), Cz = sqr(T.z), J = sqr(T.x);
    const Fp2 E = mul(C.b3, Cz);          // 3 b' Z^2
    const Fp2 F = add(add(E, E), E);      // 9 b' Z^2
    const Fp2 H = sub(sub(sqr(add(T.y, T.z)), B), Cz);  // 2 Y Z
    const Fp12 ln = line3(H, neg(add(add(J, J), J)), sub(B, E), P);
    const Fp2 XY = mul(T.x, T.y);
    const Fp2 E2 = sqr(E), E4 = add(add(E2, E2), add(E2, E2));
    T.x = mul(add(XY, XY), sub(B, F));
    T.y = sub(sqr(add(B, F)), add(add(E4, E4), E4));  // (B + F)^2 - 12 E^2
    const Fp2 BH = mul(B, H);
    T.z = add(add(BH, BH), add(BH, BH));  // 4 Y^2 (2 Y Z)
    return ln;
}
// T <- T + Q (Q affine); the line through T and Q times lambda = X - xQ Z:
//   lambda yP - theta xP w + (theta xQ - lambda yQ) w^3, theta = Y - yQ Z
static Fp12 add_step(G2p& T, const G2a& Q, const G1a& P) {
    const Fp2 theta = sub(T.y, mul(Q.y, T.z)), lambda = sub(T.x, mul(Q.x, T.z));
    const Fp12 ln = line3(lambda, neg(theta), sub(mul(theta, Q.x), mul(lambda, Q.y)), P);
    const Fp2 Cc = sqr(theta), D = sqr(lambda);
    const Fp2 E = mul(D, lambda), F = mul(T.z, Cc), G = mul(T.x, D);
    const Fp2 H = sub(add(E, F), add(G, G));
    const Fp2 y3 = sub(mul(theta, sub(G, H)), mul(T.y, E));
    T.x = mul(lambda, H);
    T.y = y3;
    T.z = mul(T.z, E);
    return ln;
}
static G2a frob_g2(const G2a& Q) {
    const Consts& C = consts();
    return {mul(conj(Q.x), C.gamma[2]), mul(conj(Q.y), C.gamma[3]), Q.inf};
}

// prod_k f_{6t+2, Q_k}(P_k) (with the two Frobenius lines), pairs with an
// infinite point skipped (their pairing is 1)
static Fp12 multi_miller(const G1a* P, const G2a* Q, int n) {
    const Consts& C = consts();
    std::vector<G2p> T;
    std::vector<int> idx;
    for (int k = 0; k < n; k++)
        if (!P[k].inf && !Q[k].inf) {
            T.push_back({Q[k].x, Q[k].y, one2()});
            idx.push_back(k);
        }
    Fp12 f = one12();
    const int top = (int)C.naf.size() - 1;
    for (int i = top - 1; i >= 0; i--) {
        f = sqr(f);
        for (size_t j = 0; j < T.size(); j++) f = mul(f, dbl_step(T[j], P[idx[j]]));
        if (C.naf[(size_t)i] != 0) {
            for (size_t j = 0; j < T.size(); j++) {
                G2a q = Q[idx[j]];
                if (C.naf[(size_t)i] < 0) q.y = neg(q.y);
                f = mul(f, add_step(T[j], q, P[idx[j]]));
            }
        }
    }
    for (size_t j = 0; j < T.size(); j++) {
        const G2a q1 = frob_g2(Q[idx[j]]);
        G2a q2 = frob_g2(q1);
        q2.y = neg(q2.y);
        f = mul(f, add_step(T[j], q1, P[idx[j]]));
        f = mul(f, add_step(T[j], q2, P[idx[j]]));
    }
    return f;
}

static G1a load_g1(const uint64_t* w) {
    G1a p;
    std::memcpy(p.x.v, w, 32);
    std::memcpy(p.y.v, w + 4, 32);
    p.inf = zkh::is_zero(p.x) && zkh::is_zero(p.y);
    return p;
}
static G2a load_g2(const uint64_t* w) {
    G2a q;
    std::memcpy(q.x.c0.v, w, 32);
    std::memcpy(q.x.c1.v, w + 4, 32);
    std::memcpy(q.y.c0.v, w + 8, 32);
    std::memcpy(q.y.c1.v, w + 12, 32);
    q.inf = zkh::fis_zero(q.x) && zkh::fis_zero(q.y);
    return q;
}

}  // namespace zkp

// ================================================================== C ABI (pairing, verifier)
using namespace zk;

struct zk_groth16_vk {
    int num_public = 0;
    uint64_t alpha1[8], beta2[16], gamma2[16], delta2[16];
    std::vector<uint64_t> ic;  // (num_public + 1) x 8 packed affine, Montgomery
};

static int consts_ok() {
    if (!zkp::consts().ok) {
        set_error("pairing: derived final-exponentiation constants failed their check");
        return ZK_ERR_INVALID;
    }
    return ZK_OK;
}

extern "C" int zk_bn254_pairing(const void* p64, const void* q128, void* out_fp12) {
    clear_error();
    if (!p64 || !q128 || !out_fp12) return ZK_ERR_INVALID;
    ZK_TRY(consts_ok());
    const zkp::G1a P = zkp::load_g1((const uint64_t*)p64);
    const zkp::G2a Q = zkp::load_g2((const uint64_t*)q128);
    const zkp::Fp12 e = zkp::final_exp(zkp::multi_miller(&P, &Q, 1));
    std::memcpy(out_fp12, &e, sizeof e);  // c0.c0 c0.c1 c0.c2 c1.c0 c1.c1 c1.c2, each Fp2 (c0, c1)
    return ZK_OK;
}

extern "C" int zk_bn254_pairing_check(const void* p64s, const void* q128s, int n, int* holds) {
    clear_error();
    if (!holds || n < 0 || (n && (!p64s || !q128s))) return ZK_ERR_INVALID;
    ZK_TRY(consts_ok());
    std::vector<zkp::G1a> P((size_t)n);
    std::vector<zkp::G2a> Q((size_t)n);
    for (int i = 0; i < n; i++) {
        P[(size_t)i] = zkp::load_g1((const uint64_t*)p64s + (size_t)i * 8);
        Q[(size_t)i] = zkp::load_g2((const uint64_t*)q128s + (size_t)i * 16);
    }
    *holds = zkp::eq(zkp::final_exp(zkp::multi_miller(P.data(), Q.data(), n)), zkp::one12()) ? 1 : 0;
    return ZK_OK;
}

static void std_to_mont_fp(uint64_t* w, int fe_count) {
    for (int i = 0; i < fe_count; i++) {
        zkh::Fe f;
        zkh::from_std(zkh::kP, f, w + 4 * i);
        std::memcpy(w + 4 * i, f.v, 32);
    }
}

extern "C" int zk_groth16_vk_load(const char* path, zk_groth16_vk** out) {
    clear_error();
    if (!path || !out) return ZK_ERR_INVALID;
    *out = nullptr;
    FILE* f = fopen(path, "rb");
    if (!f) { set_error("vk_load: cannot open %s", path); return ZK_ERR_INVALID; }
    auto rd = [&](void* p, size_t n) { return fread(p, 1, n, f) == n; };
    zk_groth16_vk* vk = new zk_groth16_vk();
    int32_t pub = 0, nic = 0;
    bool ok = rd(&pub, 4) && pub >= 0 && pub < (1 << 28) && rd(vk->alpha1, 64) && rd(vk->beta2, 128) && rd(vk->gamma2, 128) &&
              rd(vk->delta2, 128) && rd(&nic, 4) && nic >= 0 && nic < (1 << 28);
    if (ok) {
        vk->ic.resize((size_t)nic * 8);
        ok = rd(vk->ic.data(), (size_t)nic * 64);
    }
    fclose(f);
    if (!ok) {
        set_error("vk_load: %s is not a complete vk.bin", path);
        delete vk;
        return ZK_ERR_INVALID;
    }
    vk->num_public = pub;
    std_to_mont_fp(vk->alpha1, 2);
    std_to_mont_fp(vk->beta2, 4);
    std_to_mont_fp(vk->gamma2, 4);
    std_to_mont_fp(vk->delta2, 4);
    std_to_mont_fp(vk->ic.data(), 2 * nic);
    *out = vk;
    return ZK_OK;
}

extern "C" int zk_groth16_vk_from_pk(const zk_groth16_pk* pk, zk_groth16_vk** out) {
    clear_error();
    if (!pk || !out) return ZK_ERR_INVALID;
    *out = nullptr;
    const int nic = zk_groth16_vk_points(pk, nullptr, nullptr, nullptr, nullptr, nullptr, 0);
    if (nic <= 0) {
        set_error("vk_from_pk: this proving key carries no verification key (loaded from a file)");
        return ZK_ERR_INVALID;
    }
    zk_groth16_vk* vk = new zk_groth16_vk();
    vk->ic.resize((size_t)nic * 8);
    zk_groth16_vk_points(pk, vk->alpha1, vk->beta2, vk->gamma2, vk->delta2, vk->ic.data(), nic);
    vk->num_public = nic - 1;
    *out = vk;
    return ZK_OK;
}

extern "C" void zk_groth16_vk_destroy(zk_groth16_vk* vk) { delete vk; }

extern "C" int zk_groth16_vk_num_public(const zk_groth16_vk* vk) { return vk ? vk->num_public : -1; }

// 256-byte proof -> packed Montgomery A (8 words), B (16), C (8)
static void parse_proof(const uint8_t* in, uint64_t A[8], uint64_t B[16], uint64_t C[8]) {
    uint64_t* dst[8] = {A, A + 4, B, B + 4, B + 8, B + 12, C, C + 4};
    for (int k = 0; k < 8; k++) {
        uint64_t s[4];
        std::memcpy(s, in + 32 * k, 32);
        zkh::Fe f;
        zkh::from_std(zkh::kP, f, s);
        std::memcpy(dst[k], f.v, 32);
    }
}

extern "C" int zk_groth16_verify(const zk_groth16_vk* vk, int device, const void* public_inputs, int num_public, const void* proof256,
                                 int* valid) {
    clear_error();
    if (!vk || !valid || !proof256 || num_public < 0 || (num_public && !public_inputs)) return ZK_ERR_INVALID;
    *valid = 0;
    ZK_TRY(consts_ok());
    if (num_public != vk->num_public || vk->ic.size() != (size_t)(num_public + 1) * 8) return ZK_OK;  // groth16.cu:976-980
    // vk_x = IC[0] + sum_i x_i IC[i + 1]
    uint64_t sum[8] = {0};
    if (num_public > 0) {
        if (device >= 0) {
            ZK_TRY(zk_msm_g1_host(device, nullptr, vk->ic.data() + 8, public_inputs, (size_t)num_public, sum));
        } else {  // host: the reference's own loop (scalar multiplications one by one)
            zkh::Xyzz<zkh::Fe> acc, t, p;
            zkh::set_identity(acc);
            for (int i = 0; i < num_public; i++) {
                const uint64_t* q = vk->ic.data() + (size_t)(i + 1) * 8;
                bool inf = true;
                for (int k = 0; k < 8; k++) if (q[k]) inf = false;
                if (inf) continue;
                zkh::Fe x, y, s;
                std::memcpy(x.v, q, 32);
                std::memcpy(y.v, q + 4, 32);
                zkh::from_affine(p, x, y);
                std::memcpy(s.v, (const uint64_t*)public_inputs + 4 * i, 32);
                uint64_t k_std[4];
                zkh::to_std(zkh::kR, k_std, s);
                zkh::smul(t, p, k_std);
                zkh::add(acc, t);
            }
            zkh::Fe x, y;
            if (zkh::to_affine(x, y, acc)) {
                std::memcpy(sum, x.v, 32);
                std::memcpy(sum + 4, y.v, 32);
            }
        }
    }
    uint64_t vkx[8];
    ZK_TRY(zk_g1_add_affine(vk->ic.data(), sum, vkx));
    uint64_t A[8], B[16], C[8];
    parse_proof((const uint8_t*)proof256, A, B, C);
    // e(-A, B) e(alpha, beta) e(vk_x, gamma) e(C, delta) == 1
    uint64_t P[4][8], Q[4][16];
    std::memcpy(P[0], A, 64);
    {
        zkh::Fe y;
        std::memcpy(y.v, A + 4, 32);
        if (!zkh::is_zero(y)) zkh::fsub(y, zkh::zero(), y);
        std::memcpy(P[0] + 4, y.v, 32);
    }
    std::memcpy(P[1], vk->alpha1, 64);
    std::memcpy(P[2], vkx, 64);
    std::memcpy(P[3], C, 64);
    std::memcpy(Q[0], B, 128);
    std::memcpy(Q[1], vk->beta2, 128);
    std::memcpy(Q[2], vk->gamma2, 128);
    std::memcpy(Q[3], vk->delta2, 128);
    return zk_bn254_pairing_check(P, Q, 4, valid);
}
