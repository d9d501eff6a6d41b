// curve.cuh -- BN254 G1 (y^2 = x^3 + 3 over Fp) and G2 (the D-type twist over
// Fp2) point arithmetic for the MSM kernels.
//
// Buckets are kept in extended Jacobian "XYZZ" coordinates (X, Y, ZZ, ZZZ) with
// x = X/ZZ, y = Y/ZZZ and ZZ^3 = ZZZ^2 (Cohen, Miyaji & Ono 1998; formulas
// madd-2008-s, add-2008-s, dbl-2008-s-1 and mdbl-2008-s of the Explicit-Formulas
// Database).  A mixed bucket addition costs 8M + 2S, against 8M + 3S for the
// reference's Jacobian add_affine (src/curve/g1.cuh:163-189); G2 replaces the
// reference's affine-with-inversion additions (src/curve/g2.cuh:103-146) by
// the same XYZZ formulas over Fp2.  The identity is ZZ = ZZZ = 0.
//
// Affine inputs use the packed device layout x || y (64 B for G1, 128 B for
// G2); the point at infinity is the all-zero record, which is not on either
// curve, so it cannot be confused with a real point.
#pragma once
#include "field.cuh"

namespace zk {

// Rarely taken paths (doubling when a bucket meets the same point again) are
// kept out of line unless ZK_RARE_INLINE=1, so the common mixed-addition path
// stays compact in the instruction cache.
#ifndef ZK_RARE_INLINE
#define ZK_RARE_INLINE 0
#endif
#if ZK_RARE_INLINE
#define ZK_RARE __forceinline__
#else
#define ZK_RARE __noinline__
#endif

template <class F>
struct Affine {
    F x, y;
};

template <class F>
struct Xyzz {
    F x, y, zz, zzz;
};

template <class F>
__device__ __forceinline__ void set_identity(Xyzz<F>& p) {
    fset_zero(p.x); fset_one(p.y); fset_zero(p.zz); fset_zero(p.zzz);
}
template <class F>
__device__ __forceinline__ bool is_identity(const Xyzz<F>& p) { return fis_zero(p.zz); }

template <class F>
__device__ __forceinline__ void from_affine(Xyzz<F>& r, const Affine<F>& a) {
    r.x = a.x; r.y = a.y; fset_one(r.zz); fset_one(r.zzz);
}

// r = 2 * (x, y) for an affine point (mdbl-2008-s)
template <class F>
__device__ ZK_RARE void mdbl(Xyzz<F>& r, const Affine<F>& a) {
    F u, v, w, s, m, t;
    fdbl(u, a.y);            // U = 2Y
    fsqr(v, u);              // V = U^2
    fmul(w, u, v);           // W = U V
    fmul(s, a.x, v);         // S = X V
    fsqr(m, a.x);
    fadd(t, m, m);
    fadd(m, t, m);           // M = 3 X^2
    fsqr(t, m);
    fsub(t, t, s);
    fsub(r.x, t, s);         // X3 = M^2 - 2S
    fsub(t, s, r.x);
    fmul(t, m, t);
    fmul(s, w, a.y);
    fsub(r.y, t, s);         // Y3 = M (S - X3) - W Y
    r.zz = v;
    r.zzz = w;
}

// r = 2 p (dbl-2008-s-1, a = 0); identity maps to identity
template <class F>
__device__ ZK_RARE void dbl(Xyzz<F>& r, const Xyzz<F>& p) {
    if (is_identity(p)) { r = p; return; }
    F u, v, w, s, m, t;
    fdbl(u, p.y);            // U = 2 Y1
    fsqr(v, u);              // V = U^2
    fmul(w, u, v);           // W = U V
    fmul(s, p.x, v);         // S = X1 V
    fsqr(m, p.x);
    fadd(t, m, m);
    fadd(m, t, m);           // M = 3 X1^2
    fsqr(t, m);
    fsub(t, t, s);
    F x3;
    fsub(x3, t, s);          // X3 = M^2 - 2S
    fsub(t, s, x3);
    fmulsub(r.y, m, t, w, p.y);  // Y3 = M (S - X3) - W Y1, one reduction
    fmul(r.zz, v, p.zz);     // ZZ3 = V ZZ1
    fmul(r.zzz, w, p.zzz);   // ZZZ3 = W ZZZ1
    r.x = x3;
}

// acc += a, a affine and not the identity (madd-2008-s)
template <class F>
__device__ __forceinline__ void madd(Xyzz<F>& acc, const Affine<F>& a) {
    if (is_identity(acc)) { from_affine(acc, a); return; }
    F u2, s2, p, r, pp, ppp, q, t;
    fmul(u2, a.x, acc.zz);   // U2 = X2 ZZ1
    fmul(s2, a.y, acc.zzz);  // S2 = Y2 ZZZ1
    fsub(p, u2, acc.x);      // P = U2 - X1
    fsub(r, s2, acc.y);      // R = S2 - Y1
    if (fis_zero(p)) {
        if (fis_zero(r)) { mdbl(acc, a); return; }
        set_identity(acc);
        return;
    }
    fsqr(pp, p);             // PP = P^2
    fmul(ppp, p, pp);        // PPP = P PP
    fmul(q, acc.x, pp);      // Q = X1 PP
    fsqr(t, r);
    fsub(t, t, ppp);
    fsub(t, t, q);
    fsub(t, t, q);           // X3 = R^2 - PPP - 2Q
    fsub(q, q, t);
    fmulsub(acc.y, r, q, acc.y, ppp);  // Y3 = R (Q - X3) - Y1 PPP, one reduction
    acc.x = t;
    fmul(acc.zz, acc.zz, pp);     // ZZ3 = ZZ1 PP
    fmul(acc.zzz, acc.zzz, ppp);  // ZZZ3 = ZZZ1 PPP
}

// acc += b (add-2008-s), both XYZZ
template <class F>
__device__ __forceinline__ void add(Xyzz<F>& acc, const Xyzz<F>& b) {
    if (is_identity(b)) return;
    if (is_identity(acc)) { acc = b; return; }
    F u1, u2, s1, s2, p, r, pp, ppp, q, t;
    fmul(u1, acc.x, b.zz);   // U1 = X1 ZZ2
    fmul(u2, b.x, acc.zz);   // U2 = X2 ZZ1
    fmul(s1, acc.y, b.zzz);  // S1 = Y1 ZZZ2
    fmul(s2, b.y, acc.zzz);  // S2 = Y2 ZZZ1
    fsub(p, u2, u1);
    fsub(r, s2, s1);
    if (fis_zero(p)) {
        if (fis_zero(r)) { Xyzz<F> d; dbl(d, acc); acc = d; return; }
        set_identity(acc);
        return;
    }
    fsqr(pp, p);
    fmul(ppp, p, pp);
    fmul(q, u1, pp);         // Q = U1 PP
    fsqr(t, r);
    fsub(t, t, ppp);
    fsub(t, t, q);
    fsub(t, t, q);           // X3
    fsub(q, q, t);
    fmulsub(acc.y, r, q, s1, ppp);  // Y3 = R (Q - X3) - S1 PPP, one reduction
    acc.x = t;
    fmul(acc.zz, acc.zz, b.zz);
    fmul(acc.zz, acc.zz, pp);     // ZZ3 = ZZ1 ZZ2 PP
    fmul(acc.zzz, acc.zzz, b.zzz);
    fmul(acc.zzz, acc.zzz, ppp);  // ZZZ3 = ZZZ1 ZZZ2 PPP
}

// ------------------------------------------------------------ curve traits
struct G1 {
    using F = Fp;
    static constexpr int kAffineBytes = 64;
    static constexpr int kXyzzBytes = 128;
    // Resident 128-thread blocks per SM the bucket-accumulate kernel is
    // compiled for: 5 caps it at 96 registers (32 bytes spilled to local
    // memory), which runs 1.6% faster than the uncapped 120 at 4 blocks.
    static constexpr int kAccumulateMinBlocks = 5;
};
struct G2 {
    using F = Fp2;
    static constexpr int kAffineBytes = 128;
    static constexpr int kXyzzBytes = 256;
    // Fp2 arithmetic needs ~210 registers; any cap spills heavily.
    static constexpr int kAccumulateMinBlocks = 1;
};

template <class F>
__device__ __forceinline__ void load_affine(Affine<F>& a, const void* p) {
    fload_nc(a.x, p);
    fload_nc(a.y, reinterpret_cast<const char*>(p) + sizeof(F));
}
template <class F>
__device__ __forceinline__ void load_xyzz(Xyzz<F>& a, const void* p) {
    const char* c = reinterpret_cast<const char*>(p);
    fload(a.x, c);
    fload(a.y, c + sizeof(F));
    fload(a.zz, c + 2 * sizeof(F));
    fload(a.zzz, c + 3 * sizeof(F));
}
template <class F>
__device__ __forceinline__ void store_xyzz(void* p, const Xyzz<F>& a) {
    char* c = reinterpret_cast<char*>(p);
    fstore(c, a.x);
    fstore(c + sizeof(F), a.y);
    fstore(c + 2 * sizeof(F), a.zz);
    fstore(c + 3 * sizeof(F), a.zzz);
}

}  // namespace zk
