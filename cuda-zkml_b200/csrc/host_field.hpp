// host_field.hpp -- BN254 arithmetic on the host, used by the runtime for the
// few serial steps that are latency-bound on a single GPU thread: the final
// Pippenger window combine (the reference does the same on the host,
// src/msm/msm.cu:423-430), XYZZ -> affine normalisation, and layout
// conversions.  4 x 64-bit CIOS Montgomery with unsigned __int128.
#pragma once
#include <cstdint>
#include <cstring>

namespace zkh {

typedef unsigned __int128 u128;

struct Mod {
    uint64_t m[4];
    uint64_t inv;
    uint64_t one[4];
    uint64_t r2[4];
};

// BN254 p and r with their Montgomery constants (R = 2^256)
static const Mod kP = {{0x3C208C16D87CFD47ULL, 0x97816A916871CA8DULL, 0xB85045B68181585DULL, 0x30644E72E131A029ULL},
                       0x87D20782E4866389ULL,
                       {0xD35D438DC58F0D9DULL, 0x0A78EB28F5C70B3DULL, 0x666EA36F7879462CULL, 0x0E0A77C19A07DF2FULL},
                       {0xF32CFC5B538AFA89ULL, 0xB5E71911D44501FBULL, 0x47AB1EFF0A417FF6ULL, 0x06D89F71CAB8351FULL}};
static const Mod kR = {{0x43E1F593F0000001ULL, 0x2833E84879B97091ULL, 0xB85045B68181585DULL, 0x30644E72E131A029ULL},
                       0xC2E1F593EFFFFFFFULL,
                       {0xAC96341C4FFFFFFBULL, 0x36FC76959F60CD29ULL, 0x666EA36F7879462EULL, 0x0E0A77C19A07DF2FULL},
                       {0x1BB8E645AE216DA7ULL, 0x53FE3AB1E35C59E3ULL, 0x8C49833D53BB8085ULL, 0x0216D0B17F4E44A5ULL}};

struct Fe {
    uint64_t v[4];
};

inline bool is_zero(const Fe& a) { return (a.v[0] | a.v[1] | a.v[2] | a.v[3]) == 0; }
inline bool eq(const Fe& a, const Fe& b) { return std::memcmp(a.v, b.v, 32) == 0; }

inline void mul(const Mod& M, Fe& r, const Fe& a, const Fe& b) {
    uint64_t t[5] = {0, 0, 0, 0, 0};
    for (int i = 0; i < 4; i++) {
        u128 c = 0;
        for (int j = 0; j < 4; j++) {
            c += (u128)a.v[i] * b.v[j] + t[j];
            t[j] = (uint64_t)c;
            c >>= 64;
        }
        c += t[4];
        t[4] = (uint64_t)c;
        uint64_t q = t[0] * M.inv;
        c = ((u128)q * M.m[0] + t[0]) >> 64;
        for (int j = 1; j < 4; j++) {
            c += (u128)q * M.m[j] + t[j];
            t[j - 1] = (uint64_t)c;
            c >>= 64;
        }
        c += t[4];
        t[3] = (uint64_t)c;
        t[4] = (uint64_t)(c >> 64);
    }
    uint64_t u[4], br = 0;
    for (int i = 0; i < 4; i++) {
        u128 d = (u128)t[i] - M.m[i] - br;
        u[i] = (uint64_t)d;
        br = (uint64_t)(d >> 64) & 1;
    }
    if (t[4] || !br) std::memcpy(r.v, u, 32);
    else std::memcpy(r.v, t, 32);
}
inline void add(const Mod& M, Fe& r, const Fe& a, const Fe& b) {
    uint64_t t[4], u[4];
    u128 c = 0;
    for (int i = 0; i < 4; i++) { c += (u128)a.v[i] + b.v[i]; t[i] = (uint64_t)c; c >>= 64; }
    uint64_t br = 0;
    for (int i = 0; i < 4; i++) {
        u128 d = (u128)t[i] - M.m[i] - br;
        u[i] = (uint64_t)d;
        br = (uint64_t)(d >> 64) & 1;
    }
    if (c || !br) std::memcpy(r.v, u, 32);
    else std::memcpy(r.v, t, 32);
}
inline void sub(const Mod& M, Fe& r, const Fe& a, const Fe& b) {
    uint64_t t[4], br = 0;
    for (int i = 0; i < 4; i++) {
        u128 d = (u128)a.v[i] - b.v[i] - br;
        t[i] = (uint64_t)d;
        br = (uint64_t)(d >> 64) & 1;
    }
    if (br) {
        u128 c = 0;
        for (int i = 0; i < 4; i++) { c += (u128)t[i] + M.m[i]; t[i] = (uint64_t)c; c >>= 64; }
    }
    std::memcpy(r.v, t, 32);
}
inline Fe one(const Mod& M) { Fe r; std::memcpy(r.v, M.one, 32); return r; }
inline Fe zero() { Fe r = {{0, 0, 0, 0}}; return r; }
inline void pow(const Mod& M, Fe& r, const Fe& a, const uint64_t e[4]) {
    Fe acc = one(M), base = a;
    for (int bit = 255; bit >= 0; bit--) {
        mul(M, acc, acc, acc);
        if ((e[bit >> 6] >> (bit & 63)) & 1) mul(M, acc, acc, base);
    }
    r = acc;
}
inline void inv(const Mod& M, Fe& r, const Fe& a) {
    uint64_t e[4];
    std::memcpy(e, M.m, 32);
    e[0] -= 2;  // m is odd and > 2: no borrow
    pow(M, r, a, e);
}
inline void from_std(const Mod& M, Fe& r, const uint64_t s[4]) {
    Fe a;
    std::memcpy(a.v, s, 32);
    Fe r2;
    std::memcpy(r2.v, M.r2, 32);
    mul(M, r, a, r2);
}
inline void to_std(const Mod& M, uint64_t s[4], const Fe& a) {
    Fe o = {{1, 0, 0, 0}}, r;
    mul(M, r, a, o);
    std::memcpy(s, r.v, 32);
}

// ---------------------------------------------------------------- Fp / Fp2 wrappers
struct Fp {
    Fe a;
};
struct Fp2 {
    Fe c0, c1;
};

inline void fmul(Fe& r, const Fe& a, const Fe& b) { mul(kP, r, a, b); }
inline void fadd(Fe& r, const Fe& a, const Fe& b) { add(kP, r, a, b); }
inline void fsub(Fe& r, const Fe& a, const Fe& b) { sub(kP, r, a, b); }
inline void fsqr(Fe& r, const Fe& a) { mul(kP, r, a, a); }
inline void finv(Fe& r, const Fe& a) { inv(kP, r, a); }
inline bool fis_zero(const Fe& a) { return is_zero(a); }
inline void fset_one(Fe& r) { r = one(kP); }
inline void fset_zero(Fe& r) { r = zero(); }

inline void fmul(Fp2& r, const Fp2& a, const Fp2& b) {
    Fe t0, t1, s0, s1;
    fmul(t0, a.c0, b.c0);
    fmul(t1, a.c1, b.c1);
    fadd(s0, a.c0, a.c1);
    fadd(s1, b.c0, b.c1);
    fmul(s0, s0, s1);
    fsub(r.c0, t0, t1);
    fsub(s0, s0, t0);
    fsub(r.c1, s0, t1);
}
inline void fadd(Fp2& r, const Fp2& a, const Fp2& b) { fadd(r.c0, a.c0, b.c0); fadd(r.c1, a.c1, b.c1); }
inline void fsub(Fp2& r, const Fp2& a, const Fp2& b) { fsub(r.c0, a.c0, b.c0); fsub(r.c1, a.c1, b.c1); }
inline void fsqr(Fp2& r, const Fp2& a) { fmul(r, a, a); }
inline bool fis_zero(const Fp2& a) { return is_zero(a.c0) && is_zero(a.c1); }
inline void fset_one(Fp2& r) { r.c0 = one(kP); r.c1 = zero(); }
inline void fset_zero(Fp2& r) { r.c0 = zero(); r.c1 = zero(); }
inline void finv(Fp2& r, const Fp2& a) {
    // (a0 + a1 u)^-1 = (a0 - a1 u) / (a0^2 + a1^2)
    Fe n, t, ni;
    fmul(n, a.c0, a.c0);
    fmul(t, a.c1, a.c1);
    fadd(n, n, t);
    finv(ni, n);
    fmul(r.c0, a.c0, ni);
    fmul(t, a.c1, ni);
    fsub(r.c1, zero(), t);
}

// ---------------------------------------------------------------- XYZZ points
template <class F>
struct Xyzz {
    F x, y, zz, zzz;
};

template <class F>
inline void set_identity(Xyzz<F>& p) { fset_zero(p.x); fset_one(p.y); fset_zero(p.zz); fset_zero(p.zzz); }
template <class F>
inline bool is_identity(const Xyzz<F>& p) { return fis_zero(p.zz); }

template <class F>
inline void dbl(Xyzz<F>& r, const Xyzz<F>& p) {
    if (is_identity(p)) { r = p; return; }
    F u, v, w, s, m, t, x3;
    fadd(u, p.y, p.y);
    fsqr(v, u);
    fmul(w, u, v);
    fmul(s, p.x, v);
    fsqr(m, p.x);
    fadd(t, m, m);
    fadd(m, t, m);
    fsqr(t, m);
    fsub(t, t, s);
    fsub(x3, t, s);
    fsub(t, s, x3);
    fmul(t, m, t);
    fmul(s, w, p.y);
    fsub(r.y, t, s);
    fmul(r.zz, v, p.zz);
    fmul(r.zzz, w, p.zzz);
    r.x = x3;
}

template <class F>
inline void add(Xyzz<F>& acc, const Xyzz<F>& b) {
    if (is_identity(b)) return;
    if (is_identity(acc)) { acc = b; return; }
    F u1, u2, s1, s2, p, r, pp, ppp, q, t;
    fmul(u1, acc.x, b.zz);
    fmul(u2, b.x, acc.zz);
    fmul(s1, acc.y, b.zzz);
    fmul(s2, b.y, acc.zzz);
    fsub(p, u2, u1);
    fsub(r, s2, s1);
    if (fis_zero(p)) {
        if (fis_zero(r)) { Xyzz<F> d; dbl(d, acc); acc = d; return; }
        set_identity(acc);
        return;
    }
    fsqr(pp, p);
    fmul(ppp, p, pp);
    fmul(q, u1, pp);
    fsqr(t, r);
    fsub(t, t, ppp);
    fsub(t, t, q);
    fsub(t, t, q);
    fsub(q, q, t);
    fmul(q, r, q);
    fmul(s1, s1, ppp);
    fsub(acc.y, q, s1);
    acc.x = t;
    fmul(acc.zz, acc.zz, b.zz);
    fmul(acc.zz, acc.zz, pp);
    fmul(acc.zzz, acc.zzz, b.zzz);
    fmul(acc.zzz, acc.zzz, ppp);
}

// affine (x, y); returns false for the identity
template <class F>
inline bool to_affine(F& x, F& y, const Xyzz<F>& p) {
    if (is_identity(p)) { fset_zero(x); fset_zero(y); return false; }
    // x = X / ZZ, y = Y / ZZZ
    F zi, zzi;
    finv(zi, p.zz);
    fmul(x, p.x, zi);
    finv(zzi, p.zzz);
    fmul(y, p.y, zzi);
    return true;
}

template <class F>
inline void from_affine(Xyzz<F>& r, const F& x, const F& y) {
    r.x = x; r.y = y; fset_one(r.zz); fset_one(r.zzz);
}

// k * P by left-to-right double-and-add over the standard-form bits of k
template <class F>
inline void smul(Xyzz<F>& r, const Xyzz<F>& p, const uint64_t k_std[4]) {
    Xyzz<F> acc, d;
    set_identity(acc);
    for (int bit = 255; bit >= 0; bit--) {
        dbl(d, acc);
        acc = d;
        if ((k_std[bit >> 6] >> (bit & 63)) & 1) add(acc, p);
    }
    r = acc;
}

}  // namespace zkh
