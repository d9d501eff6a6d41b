// field.cuh -- BN254 Fp / Fr / Fp2 arithmetic for sm_100a.
//
// Elements are 8 x 32-bit little-endian limbs in Montgomery form (R = 2^256),
// bit-identical to the reference's 4 x 64-bit host layout
// (src/field/fp.cuh:30-34, :322-323), so a buffer of reference Fr/Fp values is a
// buffer of these.  Every operation returns the canonical residue in [0, m), as
// the reference does (single conditional subtraction, fp.cuh:417-426), which is
// what makes every downstream result bit-exact regardless of evaluation order.
//
// Multiplication is CIOS Montgomery (Koc, Acar & Kaliski, "Analyzing and
// comparing Montgomery multiplication algorithms", IEEE Micro 1996) on 32-bit
// limbs.  Each row "T += a_i * B" is issued as two PTX carry chains: the low
// halves (mad.lo.cc) into T[0..7] and the high halves (mad.hi.cc) into T[1..8].
// Both chains are complete multi-word additions, so no carry crosses an asm
// statement.  With m < 2^254 the accumulator stays below 2^288 (9 words) and
// below 2m after each shift, so one final conditional subtraction suffices.
#pragma once
#include <cstdint>

namespace zk {

// Moduli as constexpr accessors (usable in host and device code, folded to
// immediates once the limb loops are unrolled).
#define ZK_LIMBS8(name, a0, a1, a2, a3, a4, a5, a6, a7)                                   \
    __host__ __device__ static constexpr uint32_t name(int i) {                           \
        return i == 0 ? a0 : i == 1 ? a1 : i == 2 ? a2 : i == 3 ? a3 : i == 4 ? a4 : i == 5 ? a5 : i == 6 ? a6 : a7; \
    }

struct ModP {  // BN254 base field p
    ZK_LIMBS8(m, 0xD87CFD47u, 0x3C208C16u, 0x6871CA8Du, 0x97816A91u, 0x8181585Du, 0xB85045B6u, 0xE131A029u, 0x30644E72u)
    ZK_LIMBS8(one, 0xC58F0D9Du, 0xD35D438Du, 0xF5C70B3Du, 0x0A78EB28u, 0x7879462Cu, 0x666EA36Fu, 0x9A07DF2Fu, 0x0E0A77C1u)
    ZK_LIMBS8(r2, 0x538AFA89u, 0xF32CFC5Bu, 0xD44501FBu, 0xB5E71911u, 0x0A417FF6u, 0x47AB1EFFu, 0xCAB8351Fu, 0x06D89F71u)
    static constexpr uint32_t inv = 0xE4866389u;  // -p^-1 mod 2^32
};

struct ModR {  // BN254 scalar field r
    ZK_LIMBS8(m, 0xF0000001u, 0x43E1F593u, 0x79B97091u, 0x2833E848u, 0x8181585Du, 0xB85045B6u, 0xE131A029u, 0x30644E72u)
    ZK_LIMBS8(one, 0x4FFFFFFBu, 0xAC96341Cu, 0x9F60CD29u, 0x36FC7695u, 0x7879462Eu, 0x666EA36Fu, 0x9A07DF2Fu, 0x0E0A77C1u)
    ZK_LIMBS8(r2, 0xAE216DA7u, 0x1BB8E645u, 0xE35C59E3u, 0x53FE3AB1u, 0x53BB8085u, 0x8C49833Du, 0x7F4E44A5u, 0x0216D0B1u)
    static constexpr uint32_t inv = 0xEFFFFFFFu;  // -r^-1 mod 2^32
};

template <class M>
struct Fe {
    uint32_t v[8];
};
using Fp = Fe<ModP>;
using Fr = Fe<ModR>;

// --------------------------------------------------------------- limb rows
// t[0..8] += a * b[0..7]   (caller guarantees no carry out of t[8])
//
// ZK_ROW_PAIRED=1 (default): the low and high halves of each product a*b_j
// are adjacent in one carry chain.  Products with even j land on words
// (j, j+1) = 0..7, so they form one contiguous chain; products with odd j
// land on words 1..8 and form a second one.  ZK_ROW_PAIRED=0: one chain of
// all low halves (words 0..7) then one of all high halves (words 1..8).
#ifndef ZK_ROW_PAIRED
#define ZK_ROW_PAIRED 1
#endif

__device__ __forceinline__ void mac_row(uint32_t& t0, uint32_t& t1, uint32_t& t2, uint32_t& t3,
                                        uint32_t& t4, uint32_t& t5, uint32_t& t6, uint32_t& t7,
                                        uint32_t& t8, uint32_t a, const uint32_t* b) {
#if ZK_ROW_PAIRED
    asm("mad.lo.cc.u32  %0, %9, %10, %0;\n\t"
        "madc.hi.cc.u32 %1, %9, %10, %1;\n\t"
        "madc.lo.cc.u32 %2, %9, %12, %2;\n\t"
        "madc.hi.cc.u32 %3, %9, %12, %3;\n\t"
        "madc.lo.cc.u32 %4, %9, %14, %4;\n\t"
        "madc.hi.cc.u32 %5, %9, %14, %5;\n\t"
        "madc.lo.cc.u32 %6, %9, %16, %6;\n\t"
        "madc.hi.cc.u32 %7, %9, %16, %7;\n\t"
        "addc.u32       %8, %8, 0;\n\t"
        "mad.lo.cc.u32  %1, %9, %11, %1;\n\t"
        "madc.hi.cc.u32 %2, %9, %11, %2;\n\t"
        "madc.lo.cc.u32 %3, %9, %13, %3;\n\t"
        "madc.hi.cc.u32 %4, %9, %13, %4;\n\t"
        "madc.lo.cc.u32 %5, %9, %15, %5;\n\t"
        "madc.hi.cc.u32 %6, %9, %15, %6;\n\t"
        "madc.lo.cc.u32 %7, %9, %17, %7;\n\t"
        "madc.hi.u32    %8, %9, %17, %8;"
        : "+r"(t0), "+r"(t1), "+r"(t2), "+r"(t3), "+r"(t4), "+r"(t5), "+r"(t6), "+r"(t7), "+r"(t8)
        : "r"(a), "r"(b[0]), "r"(b[1]), "r"(b[2]), "r"(b[3]), "r"(b[4]), "r"(b[5]), "r"(b[6]),
          "r"(b[7]));
#else
    asm("mad.lo.cc.u32  %0, %9, %10, %0;\n\t"
        "madc.lo.cc.u32 %1, %9, %11, %1;\n\t"
        "madc.lo.cc.u32 %2, %9, %12, %2;\n\t"
        "madc.lo.cc.u32 %3, %9, %13, %3;\n\t"
        "madc.lo.cc.u32 %4, %9, %14, %4;\n\t"
        "madc.lo.cc.u32 %5, %9, %15, %5;\n\t"
        "madc.lo.cc.u32 %6, %9, %16, %6;\n\t"
        "madc.lo.cc.u32 %7, %9, %17, %7;\n\t"
        "addc.u32       %8, %8, 0;\n\t"
        "mad.hi.cc.u32  %1, %9, %10, %1;\n\t"
        "madc.hi.cc.u32 %2, %9, %11, %2;\n\t"
        "madc.hi.cc.u32 %3, %9, %12, %3;\n\t"
        "madc.hi.cc.u32 %4, %9, %13, %4;\n\t"
        "madc.hi.cc.u32 %5, %9, %14, %5;\n\t"
        "madc.hi.cc.u32 %6, %9, %15, %6;\n\t"
        "madc.hi.cc.u32 %7, %9, %16, %7;\n\t"
        "madc.hi.u32    %8, %9, %17, %8;"
        : "+r"(t0), "+r"(t1), "+r"(t2), "+r"(t3), "+r"(t4), "+r"(t5), "+r"(t6), "+r"(t7), "+r"(t8)
        : "r"(a), "r"(b[0]), "r"(b[1]), "r"(b[2]), "r"(b[3]), "r"(b[4]), "r"(b[5]), "r"(b[6]),
          "r"(b[7]));
#endif
}

// r = t - m if t >= m else t   (t < 2m)
template <class M>
__device__ __forceinline__ void cond_sub(uint32_t* r, const uint32_t* t) {
    uint32_t u[8], bw;
    asm("sub.cc.u32  %0, %9, %17;\n\t"
        "subc.cc.u32 %1, %10, %18;\n\t"
        "subc.cc.u32 %2, %11, %19;\n\t"
        "subc.cc.u32 %3, %12, %20;\n\t"
        "subc.cc.u32 %4, %13, %21;\n\t"
        "subc.cc.u32 %5, %14, %22;\n\t"
        "subc.cc.u32 %6, %15, %23;\n\t"
        "subc.cc.u32 %7, %16, %24;\n\t"
        "subc.u32    %8, 0, 0;"
        : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
          "=r"(u[7]), "=r"(bw)
        : "r"(t[0]), "r"(t[1]), "r"(t[2]), "r"(t[3]), "r"(t[4]), "r"(t[5]), "r"(t[6]), "r"(t[7]),
          "r"(M::m(0)), "r"(M::m(1)), "r"(M::m(2)), "r"(M::m(3)), "r"(M::m(4)), "r"(M::m(5)),
          "r"(M::m(6)), "r"(M::m(7)));
#pragma unroll
    for (int i = 0; i < 8; i++) r[i] = bw ? t[i] : u[i];
}

// --------------------------------------------------------------- Fe ops
// ZK_FMUL_OUTLINE=1 (default) compiles every multiplication as a call to one
// shared out-of-line body instead of inlining ~300 instructions at each use.
// The point-addition loops then fit the instruction cache; fully inlined, the
// MSM kernels stalled mostly on instruction fetch (measured with ncu).
#ifndef ZK_FMUL_OUTLINE
#define ZK_FMUL_OUTLINE 1
#endif

template <class M>
__device__ __forceinline__ void fmul_inline(Fe<M>& r, const Fe<M>& a, const Fe<M>& b) {
    uint32_t t0 = 0, t1 = 0, t2 = 0, t3 = 0, t4 = 0, t5 = 0, t6 = 0, t7 = 0, t8 = 0;
    constexpr uint32_t mm[8] = {M::m(0), M::m(1), M::m(2), M::m(3), M::m(4), M::m(5), M::m(6), M::m(7)};
#pragma unroll
    for (int i = 0; i < 8; i++) {
        mac_row(t0, t1, t2, t3, t4, t5, t6, t7, t8, a.v[i], b.v);
        uint32_t q = t0 * M::inv;
        mac_row(t0, t1, t2, t3, t4, t5, t6, t7, t8, q, mm);
        // t0 == 0 now: shift down one word
        t0 = t1; t1 = t2; t2 = t3; t3 = t4; t4 = t5; t5 = t6; t6 = t7; t7 = t8; t8 = 0;
    }
    uint32_t t[8] = {t0, t1, t2, t3, t4, t5, t6, t7};
    cond_sub<M>(r.v, t);
}

template <class M>
__device__ __noinline__ Fe<M> fmul_outline(Fe<M> a, Fe<M> b) {
    Fe<M> r;
    fmul_inline(r, a, b);
    return r;
}

template <class M>
__device__ __forceinline__ void fmul(Fe<M>& r, const Fe<M>& a, const Fe<M>& b) {
#if ZK_FMUL_OUTLINE
    r = fmul_outline<M>(a, b);
#else
    fmul_inline(r, a, b);
#endif
}

// r = a^2 (Montgomery): the product part computes each off-diagonal a_i a_j once
// (28 products, doubled) plus the 8 diagonal squares into a 16-word T, then a
// separate reduction slides a 10-word window over T (8 reduction rows; a carry
// word catches the window's overflow).  616 instead of 784 FMA-heavy cycles per
// warp for a Montgomery product.  Every carry chain ends in a word the partial
// value provably does not overflow: after off-diagonal row i the sum is below
// 2^(32 (i + 9)), a^2 < 2^512, and the result (a^2 + Q m) / R < 2 m.
template <class M>
__device__ __forceinline__ void fsqr_inline(Fe<M>& r, const Fe<M>& a) {
    uint32_t T[16];
#pragma unroll
    for (int k = 0; k < 16; k++) T[k] = 0;
    // off-diagonal row 0: T[1..8] += a_0 * a[1..7]
    asm("mad.lo.cc.u32  %0, %8, %9, %0;\n\t"
        "madc.lo.cc.u32 %1, %8, %10, %1;\n\t"
        "madc.lo.cc.u32 %2, %8, %11, %2;\n\t"
        "madc.lo.cc.u32 %3, %8, %12, %3;\n\t"
        "madc.lo.cc.u32 %4, %8, %13, %4;\n\t"
        "madc.lo.cc.u32 %5, %8, %14, %5;\n\t"
        "madc.lo.cc.u32 %6, %8, %15, %6;\n\t"
        "addc.u32       %7, %7, 0;\n\t"
        "mad.hi.cc.u32  %1, %8, %9, %1;\n\t"
        "madc.hi.cc.u32 %2, %8, %10, %2;\n\t"
        "madc.hi.cc.u32 %3, %8, %11, %3;\n\t"
        "madc.hi.cc.u32 %4, %8, %12, %4;\n\t"
        "madc.hi.cc.u32 %5, %8, %13, %5;\n\t"
        "madc.hi.cc.u32 %6, %8, %14, %6;\n\t"
        "madc.hi.u32    %7, %8, %15, %7;"
        : "+r"(T[1]), "+r"(T[2]), "+r"(T[3]), "+r"(T[4]), "+r"(T[5]), "+r"(T[6]), "+r"(T[7]), "+r"(T[8])
        : "r"(a.v[0]), "r"(a.v[1]), "r"(a.v[2]), "r"(a.v[3]), "r"(a.v[4]), "r"(a.v[5]), "r"(a.v[6]), "r"(a.v[7]));
    // off-diagonal row 1: T[3..9] += a_1 * a[2..7]
    asm("mad.lo.cc.u32  %0, %7, %8, %0;\n\t"
        "madc.lo.cc.u32 %1, %7, %9, %1;\n\t"
        "madc.lo.cc.u32 %2, %7, %10, %2;\n\t"
        "madc.lo.cc.u32 %3, %7, %11, %3;\n\t"
        "madc.lo.cc.u32 %4, %7, %12, %4;\n\t"
        "madc.lo.cc.u32 %5, %7, %13, %5;\n\t"
        "addc.u32       %6, %6, 0;\n\t"
        "mad.hi.cc.u32  %1, %7, %8, %1;\n\t"
        "madc.hi.cc.u32 %2, %7, %9, %2;\n\t"
        "madc.hi.cc.u32 %3, %7, %10, %3;\n\t"
        "madc.hi.cc.u32 %4, %7, %11, %4;\n\t"
        "madc.hi.cc.u32 %5, %7, %12, %5;\n\t"
        "madc.hi.u32    %6, %7, %13, %6;"
        : "+r"(T[3]), "+r"(T[4]), "+r"(T[5]), "+r"(T[6]), "+r"(T[7]), "+r"(T[8]), "+r"(T[9])
        : "r"(a.v[1]), "r"(a.v[2]), "r"(a.v[3]), "r"(a.v[4]), "r"(a.v[5]), "r"(a.v[6]), "r"(a.v[7]));
    // off-diagonal row 2: T[5..10] += a_2 * a[3..7]
    asm("mad.lo.cc.u32  %0, %6, %7, %0;\n\t"
        "madc.lo.cc.u32 %1, %6, %8, %1;\n\t"
        "madc.lo.cc.u32 %2, %6, %9, %2;\n\t"
        "madc.lo.cc.u32 %3, %6, %10, %3;\n\t"
        "madc.lo.cc.u32 %4, %6, %11, %4;\n\t"
        "addc.u32       %5, %5, 0;\n\t"
        "mad.hi.cc.u32  %1, %6, %7, %1;\n\t"
        "madc.hi.cc.u32 %2, %6, %8, %2;\n\t"
        "madc.hi.cc.u32 %3, %6, %9, %3;\n\t"
        "madc.hi.cc.u32 %4, %6, %10, %4;\n\t"
        "madc.hi.u32    %5, %6, %11, %5;"
        : "+r"(T[5]), "+r"(T[6]), "+r"(T[7]), "+r"(T[8]), "+r"(T[9]), "+r"(T[10])
        : "r"(a.v[2]), "r"(a.v[3]), "r"(a.v[4]), "r"(a.v[5]), "r"(a.v[6]), "r"(a.v[7]));
    // off-diagonal row 3: T[7..11] += a_3 * a[4..7]
    asm("mad.lo.cc.u32  %0, %5, %6, %0;\n\t"
        "madc.lo.cc.u32 %1, %5, %7, %1;\n\t"
        "madc.lo.cc.u32 %2, %5, %8, %2;\n\t"
        "madc.lo.cc.u32 %3, %5, %9, %3;\n\t"
        "addc.u32       %4, %4, 0;\n\t"
        "mad.hi.cc.u32  %1, %5, %6, %1;\n\t"
        "madc.hi.cc.u32 %2, %5, %7, %2;\n\t"
        "madc.hi.cc.u32 %3, %5, %8, %3;\n\t"
        "madc.hi.u32    %4, %5, %9, %4;"
        : "+r"(T[7]), "+r"(T[8]), "+r"(T[9]), "+r"(T[10]), "+r"(T[11])
        : "r"(a.v[3]), "r"(a.v[4]), "r"(a.v[5]), "r"(a.v[6]), "r"(a.v[7]));
    // off-diagonal row 4: T[9..12] += a_4 * a[5..7]
    asm("mad.lo.cc.u32  %0, %4, %5, %0;\n\t"
        "madc.lo.cc.u32 %1, %4, %6, %1;\n\t"
        "madc.lo.cc.u32 %2, %4, %7, %2;\n\t"
        "addc.u32       %3, %3, 0;\n\t"
        "mad.hi.cc.u32  %1, %4, %5, %1;\n\t"
        "madc.hi.cc.u32 %2, %4, %6, %2;\n\t"
        "madc.hi.u32    %3, %4, %7, %3;"
        : "+r"(T[9]), "+r"(T[10]), "+r"(T[11]), "+r"(T[12])
        : "r"(a.v[4]), "r"(a.v[5]), "r"(a.v[6]), "r"(a.v[7]));
    // off-diagonal row 5: T[11..13] += a_5 * a[6..7]
    asm("mad.lo.cc.u32  %0, %3, %4, %0;\n\t"
        "madc.lo.cc.u32 %1, %3, %5, %1;\n\t"
        "addc.u32       %2, %2, 0;\n\t"
        "mad.hi.cc.u32  %1, %3, %4, %1;\n\t"
        "madc.hi.u32    %2, %3, %5, %2;"
        : "+r"(T[11]), "+r"(T[12]), "+r"(T[13])
        : "r"(a.v[5]), "r"(a.v[6]), "r"(a.v[7]));
    // off-diagonal row 6: T[13..14] += a_6 * a[7..7]
    asm("mad.lo.cc.u32  %0, %2, %3, %0;\n\t"
        "addc.u32       %1, %1, 0;\n\t"
        "mad.hi.cc.u32  %1, %2, %3, %1;"
        : "+r"(T[13]), "+r"(T[14])
        : "r"(a.v[6]), "r"(a.v[7]));
    // T = 2 T
    asm("add.cc.u32  %0, %0, %0;\n\t"
        "addc.cc.u32 %1, %1, %1;\n\t"
        "addc.cc.u32 %2, %2, %2;\n\t"
        "addc.cc.u32 %3, %3, %3;\n\t"
        "addc.cc.u32 %4, %4, %4;\n\t"
        "addc.cc.u32 %5, %5, %5;\n\t"
        "addc.cc.u32 %6, %6, %6;\n\t"
        "addc.cc.u32 %7, %7, %7;\n\t"
        "addc.cc.u32 %8, %8, %8;\n\t"
        "addc.cc.u32 %9, %9, %9;\n\t"
        "addc.cc.u32 %10, %10, %10;\n\t"
        "addc.cc.u32 %11, %11, %11;\n\t"
        "addc.cc.u32 %12, %12, %12;\n\t"
        "addc.cc.u32 %13, %13, %13;\n\t"
        "addc.cc.u32 %14, %14, %14;\n\t"
        "addc.u32    %15, %15, %15;"
        : "+r"(T[0]), "+r"(T[1]), "+r"(T[2]), "+r"(T[3]), "+r"(T[4]), "+r"(T[5]), "+r"(T[6]), "+r"(T[7]), "+r"(T[8]), "+r"(T[9]), "+r"(T[10]), "+r"(T[11]), "+r"(T[12]), "+r"(T[13]), "+r"(T[14]), "+r"(T[15]));
    // T += sum a_i^2 2^(64 i)
    asm("mad.lo.cc.u32  %0, %16, %16, %0;\n\t"
        "madc.hi.cc.u32 %1, %16, %16, %1;\n\t"
        "madc.lo.cc.u32 %2, %17, %17, %2;\n\t"
        "madc.hi.cc.u32 %3, %17, %17, %3;\n\t"
        "madc.lo.cc.u32 %4, %18, %18, %4;\n\t"
        "madc.hi.cc.u32 %5, %18, %18, %5;\n\t"
        "madc.lo.cc.u32 %6, %19, %19, %6;\n\t"
        "madc.hi.cc.u32 %7, %19, %19, %7;\n\t"
        "madc.lo.cc.u32 %8, %20, %20, %8;\n\t"
        "madc.hi.cc.u32 %9, %20, %20, %9;\n\t"
        "madc.lo.cc.u32 %10, %21, %21, %10;\n\t"
        "madc.hi.cc.u32 %11, %21, %21, %11;\n\t"
        "madc.lo.cc.u32 %12, %22, %22, %12;\n\t"
        "madc.hi.cc.u32 %13, %22, %22, %13;\n\t"
        "madc.lo.cc.u32 %14, %23, %23, %14;\n\t"
        "madc.hi.u32    %15, %23, %23, %15;"
        : "+r"(T[0]), "+r"(T[1]), "+r"(T[2]), "+r"(T[3]), "+r"(T[4]), "+r"(T[5]), "+r"(T[6]), "+r"(T[7]), "+r"(T[8]), "+r"(T[9]), "+r"(T[10]), "+r"(T[11]), "+r"(T[12]), "+r"(T[13]), "+r"(T[14]), "+r"(T[15])
        : "r"(a.v[0]), "r"(a.v[1]), "r"(a.v[2]), "r"(a.v[3]), "r"(a.v[4]), "r"(a.v[5]), "r"(a.v[6]), "r"(a.v[7]));
    // reduction: window t0..t8 over T, t9 catches its carry
    uint32_t t0 = T[0], t1 = T[1], t2 = T[2], t3 = T[3], t4 = T[4], t5 = T[5], t6 = T[6], t7 = T[7], t8 = T[8], t9 = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t q = t0 * M::inv;
        asm("mad.lo.cc.u32  %0, %10, %11, %0;\n\t"
            "madc.hi.cc.u32 %1, %10, %11, %1;\n\t"
            "madc.lo.cc.u32 %2, %10, %13, %2;\n\t"
            "madc.hi.cc.u32 %3, %10, %13, %3;\n\t"
            "madc.lo.cc.u32 %4, %10, %15, %4;\n\t"
            "madc.hi.cc.u32 %5, %10, %15, %5;\n\t"
            "madc.lo.cc.u32 %6, %10, %17, %6;\n\t"
            "madc.hi.cc.u32 %7, %10, %17, %7;\n\t"
            "addc.cc.u32    %8, %8, 0;\n\t"
            "addc.u32       %9, %9, 0;\n\t"
            "mad.lo.cc.u32  %1, %10, %12, %1;\n\t"
            "madc.hi.cc.u32 %2, %10, %12, %2;\n\t"
            "madc.lo.cc.u32 %3, %10, %14, %3;\n\t"
            "madc.hi.cc.u32 %4, %10, %14, %4;\n\t"
            "madc.lo.cc.u32 %5, %10, %16, %5;\n\t"
            "madc.hi.cc.u32 %6, %10, %16, %6;\n\t"
            "madc.lo.cc.u32 %7, %10, %18, %7;\n\t"
            "madc.hi.cc.u32 %8, %10, %18, %8;\n\t"
            "addc.u32       %9, %9, 0;"
            : "+r"(t0), "+r"(t1), "+r"(t2), "+r"(t3), "+r"(t4), "+r"(t5), "+r"(t6), "+r"(t7), "+r"(t8), "+r"(t9)
            : "r"(q), "r"(M::m(0)), "r"(M::m(1)), "r"(M::m(2)), "r"(M::m(3)), "r"(M::m(4)), "r"(M::m(5)), "r"(M::m(6)),
              "r"(M::m(7)));
        // t0 == 0: shift down one word and bring in T[i + 9]
        t0 = t1; t1 = t2; t2 = t3; t3 = t4; t4 = t5; t5 = t6; t6 = t7; t7 = t8; t8 = t9; t9 = 0;
        if (i + 9 <= 15) asm("add.cc.u32 %0, %0, %2;\n\taddc.u32 %1, 0, 0;" : "+r"(t8), "=r"(t9) : "r"(T[i + 9]));
    }
    uint32_t t[8] = {t0, t1, t2, t3, t4, t5, t6, t7};
    cond_sub<M>(r.v, t);
}

template <class M>
__device__ __noinline__ Fe<M> fsqr_outline(Fe<M> a) {
    Fe<M> r;
    fsqr_inline(r, a);
    return r;
}

template <class M>
__device__ __forceinline__ void fsqr(Fe<M>& r, const Fe<M>& a) {
#if ZK_FMUL_OUTLINE
    r = fsqr_outline<M>(a);
#else
    fsqr_inline(r, a);
#endif
}

// r = a b + c d with one Montgomery reduction: each CIOS step adds the rows a_i b
// and c_i d before its reduction row, 48 instead of 2 x 32 multiply-adds a step.
// The 9-word accumulator stays below 3 2^286 within a step (inputs < m < 2^254),
// and the result is (a b + c d + Q m) / R < m + 2 m^2 / R < 1.5 m, so one final
// conditional subtraction still gives the canonical residue.
template <class M>
__device__ __forceinline__ void fmul2sum_inline(Fe<M>& r, const Fe<M>& a, const Fe<M>& b, const Fe<M>& c, const Fe<M>& d) {
    uint32_t t0 = 0, t1 = 0, t2 = 0, t3 = 0, t4 = 0, t5 = 0, t6 = 0, t7 = 0, t8 = 0;
    constexpr uint32_t mm[8] = {M::m(0), M::m(1), M::m(2), M::m(3), M::m(4), M::m(5), M::m(6), M::m(7)};
#pragma unroll
    for (int i = 0; i < 8; i++) {
        mac_row(t0, t1, t2, t3, t4, t5, t6, t7, t8, a.v[i], b.v);
        mac_row(t0, t1, t2, t3, t4, t5, t6, t7, t8, c.v[i], d.v);
        uint32_t q = t0 * M::inv;
        mac_row(t0, t1, t2, t3, t4, t5, t6, t7, t8, q, mm);
        t0 = t1; t1 = t2; t2 = t3; t3 = t4; t4 = t5; t5 = t6; t6 = t7; t7 = t8; t8 = 0;
    }
    uint32_t t[8] = {t0, t1, t2, t3, t4, t5, t6, t7};
    cond_sub<M>(r.v, t);
}

template <class M>
__device__ __noinline__ Fe<M> fmul2sum_outline(Fe<M> a, Fe<M> b, Fe<M> c, Fe<M> d) {
    Fe<M> r;
    fmul2sum_inline(r, a, b, c, d);
    return r;
}

template <class M>
__device__ __forceinline__ void fmul2sum(Fe<M>& r, const Fe<M>& a, const Fe<M>& b, const Fe<M>& c, const Fe<M>& d) {
#if ZK_FMUL_OUTLINE
    r = fmul2sum_outline<M>(a, b, c, d);
#else
    fmul2sum_inline(r, a, b, c, d);
#endif
}

template <class M>
__device__ __forceinline__ void fadd(Fe<M>& r, const Fe<M>& a, const Fe<M>& b) {
    uint32_t t[8];
    asm("add.cc.u32  %0, %8, %16;\n\t"
        "addc.cc.u32 %1, %9, %17;\n\t"
        "addc.cc.u32 %2, %10, %18;\n\t"
        "addc.cc.u32 %3, %11, %19;\n\t"
        "addc.cc.u32 %4, %12, %20;\n\t"
        "addc.cc.u32 %5, %13, %21;\n\t"
        "addc.cc.u32 %6, %14, %22;\n\t"
        "addc.u32    %7, %15, %23;"
        : "=r"(t[0]), "=r"(t[1]), "=r"(t[2]), "=r"(t[3]), "=r"(t[4]), "=r"(t[5]), "=r"(t[6]), "=r"(t[7])
        : "r"(a.v[0]), "r"(a.v[1]), "r"(a.v[2]), "r"(a.v[3]), "r"(a.v[4]), "r"(a.v[5]), "r"(a.v[6]),
          "r"(a.v[7]), "r"(b.v[0]), "r"(b.v[1]), "r"(b.v[2]), "r"(b.v[3]), "r"(b.v[4]), "r"(b.v[5]),
          "r"(b.v[6]), "r"(b.v[7]));
    cond_sub<M>(r.v, t);
}

template <class M>
__device__ __forceinline__ void fdbl(Fe<M>& r, const Fe<M>& a) { fadd(r, a, a); }

template <class M>
__device__ __forceinline__ void fsub(Fe<M>& r, const Fe<M>& a, const Fe<M>& b) {
    uint32_t t[8], bw;
    asm("sub.cc.u32  %0, %9, %17;\n\t"
        "subc.cc.u32 %1, %10, %18;\n\t"
        "subc.cc.u32 %2, %11, %19;\n\t"
        "subc.cc.u32 %3, %12, %20;\n\t"
        "subc.cc.u32 %4, %13, %21;\n\t"
        "subc.cc.u32 %5, %14, %22;\n\t"
        "subc.cc.u32 %6, %15, %23;\n\t"
        "subc.cc.u32 %7, %16, %24;\n\t"
        "subc.u32    %8, 0, 0;"
        : "=r"(t[0]), "=r"(t[1]), "=r"(t[2]), "=r"(t[3]), "=r"(t[4]), "=r"(t[5]), "=r"(t[6]),
          "=r"(t[7]), "=r"(bw)
        : "r"(a.v[0]), "r"(a.v[1]), "r"(a.v[2]), "r"(a.v[3]), "r"(a.v[4]), "r"(a.v[5]), "r"(a.v[6]),
          "r"(a.v[7]), "r"(b.v[0]), "r"(b.v[1]), "r"(b.v[2]), "r"(b.v[3]), "r"(b.v[4]), "r"(b.v[5]),
          "r"(b.v[6]), "r"(b.v[7]));
    // add back m masked by the borrow word (0 or 0xffffffff)
    asm("add.cc.u32  %0, %0, %8;\n\t"
        "addc.cc.u32 %1, %1, %9;\n\t"
        "addc.cc.u32 %2, %2, %10;\n\t"
        "addc.cc.u32 %3, %3, %11;\n\t"
        "addc.cc.u32 %4, %4, %12;\n\t"
        "addc.cc.u32 %5, %5, %13;\n\t"
        "addc.cc.u32 %6, %6, %14;\n\t"
        "addc.u32    %7, %7, %15;"
        : "+r"(t[0]), "+r"(t[1]), "+r"(t[2]), "+r"(t[3]), "+r"(t[4]), "+r"(t[5]), "+r"(t[6]), "+r"(t[7])
        : "r"(M::m(0) & bw), "r"(M::m(1) & bw), "r"(M::m(2) & bw), "r"(M::m(3) & bw),
          "r"(M::m(4) & bw), "r"(M::m(5) & bw), "r"(M::m(6) & bw), "r"(M::m(7) & bw));
#pragma unroll
    for (int i = 0; i < 8; i++) r.v[i] = t[i];
}

template <class M>
__device__ __forceinline__ bool fis_zero(const Fe<M>& a) {
    return (a.v[0] | a.v[1] | a.v[2] | a.v[3] | a.v[4] | a.v[5] | a.v[6] | a.v[7]) == 0;
}
template <class M>
__device__ __forceinline__ void fneg(Fe<M>& r, const Fe<M>& a) {
    Fe<M> z;
#pragma unroll
    for (int i = 0; i < 8; i++) z.v[i] = 0;
    fsub(r, z, a);
}

// r = sum_{k < K} a_k b_k with one Montgomery reduction (K <= 4).  For both
// BN254 moduli m < 0.76 2^254, so within a step the accumulator stays below
// (K + 1) 2^32 m < 2^288 (9 words) and the result below m (1 + K m / R) < 1.76 m:
// one final conditional subtraction, as for a single product.
template <class M, int K>
__device__ __forceinline__ void fmulsum_inline(Fe<M>& r, const Fe<M>* a, const Fe<M>* b) {
    static_assert(K >= 1 && K <= 4, "at most four products share a reduction");
    uint32_t t0 = 0, t1 = 0, t2 = 0, t3 = 0, t4 = 0, t5 = 0, t6 = 0, t7 = 0, t8 = 0;
    constexpr uint32_t mm[8] = {M::m(0), M::m(1), M::m(2), M::m(3), M::m(4), M::m(5), M::m(6), M::m(7)};
#pragma unroll
    for (int i = 0; i < 8; i++) {
#pragma unroll
        for (int k = 0; k < K; k++) mac_row(t0, t1, t2, t3, t4, t5, t6, t7, t8, a[k].v[i], b[k].v);
        uint32_t q = t0 * M::inv;
        mac_row(t0, t1, t2, t3, t4, t5, t6, t7, t8, q, mm);
        t0 = t1; t1 = t2; t2 = t3; t3 = t4; t4 = t5; t5 = t6; t6 = t7; t7 = t8; t8 = 0;
    }
    uint32_t t[8] = {t0, t1, t2, t3, t4, t5, t6, t7};
    cond_sub<M>(r.v, t);
}

// r = a b - c d = a b + (m - c) d, one reduction
template <class M>
__device__ __forceinline__ void fmulsub(Fe<M>& r, const Fe<M>& a, const Fe<M>& b, const Fe<M>& c, const Fe<M>& d) {
    Fe<M> cn;
    fneg(cn, c);
    fmul2sum(r, a, b, cn, d);
}
template <class M>
__device__ __forceinline__ void fset_zero(Fe<M>& r) {
#pragma unroll
    for (int i = 0; i < 8; i++) r.v[i] = 0;
}
template <class M>
__device__ __forceinline__ void fset_one(Fe<M>& r) {
#pragma unroll
    for (int i = 0; i < 8; i++) r.v[i] = M::one(i);
}
template <class M>
__device__ __forceinline__ bool feq(const Fe<M>& a, const Fe<M>& b) {
    uint32_t d = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) d |= a.v[i] ^ b.v[i];
    return d == 0;
}
// standard form: a * 1 * R^-1
template <class M>
__device__ __forceinline__ void ffrom_mont(Fe<M>& r, const Fe<M>& a) {
    Fe<M> one;
    one.v[0] = 1;
#pragma unroll
    for (int i = 1; i < 8; i++) one.v[i] = 0;
    fmul(r, a, one);
}

// --------------------------------------------------------------- Fp2
// Fp2 = Fp[u]/(u^2 + 1), as src/field/fp2.cuh:22-134
struct Fp2 {
    Fp c0, c1;
};

__device__ __forceinline__ void fmul(Fp2& r, const Fp2& a, const Fp2& b) {
    Fp t0, t1, s0, s1;
    fmul(t0, a.c0, b.c0);
    fmul(t1, a.c1, b.c1);
    fadd(s0, a.c0, a.c1);
    fadd(s1, b.c0, b.c1);
    fmul(s0, s0, s1);          // (a0+a1)(b0+b1)
    fsub(r.c0, t0, t1);        // a0b0 - a1b1
    fsub(s0, s0, t0);
    fsub(r.c1, s0, t1);        // a0b1 + a1b0
}
__device__ __forceinline__ void fsqr(Fp2& r, const Fp2& a) {
    Fp s, d, m;
    fadd(s, a.c0, a.c1);
    fsub(d, a.c0, a.c1);
    fmul(m, a.c0, a.c1);
    fmul(r.c0, s, d);          // a0^2 - a1^2
    fadd(r.c1, m, m);          // 2 a0 a1
}
__device__ __forceinline__ void fadd(Fp2& r, const Fp2& a, const Fp2& b) { fadd(r.c0, a.c0, b.c0); fadd(r.c1, a.c1, b.c1); }
__device__ __forceinline__ void fsub(Fp2& r, const Fp2& a, const Fp2& b) { fsub(r.c0, a.c0, b.c0); fsub(r.c1, a.c1, b.c1); }
// r = a b - c d over Fp2 (two Karatsuba products; no shared reduction)
__device__ __forceinline__ void fmulsub(Fp2& r, const Fp2& a, const Fp2& b, const Fp2& c, const Fp2& d);
__device__ __forceinline__ void fdbl(Fp2& r, const Fp2& a) { fadd(r.c0, a.c0, a.c0); fadd(r.c1, a.c1, a.c1); }
__device__ __forceinline__ void fneg(Fp2& r, const Fp2& a) { fneg(r.c0, a.c0); fneg(r.c1, a.c1); }
__device__ __forceinline__ bool fis_zero(const Fp2& a) { return fis_zero(a.c0) && fis_zero(a.c1); }
__device__ __forceinline__ void fset_zero(Fp2& r) { fset_zero(r.c0); fset_zero(r.c1); }
__device__ __forceinline__ void fset_one(Fp2& r) { fset_one(r.c0); fset_zero(r.c1); }

// --------------------------------------------------------------- loads/stores
template <class M>
__device__ __forceinline__ void fload(Fe<M>& r, const void* p) {
    const uint4* q = reinterpret_cast<const uint4*>(p);
    uint4 a = q[0], b = q[1];
    r.v[0] = a.x; r.v[1] = a.y; r.v[2] = a.z; r.v[3] = a.w;
    r.v[4] = b.x; r.v[5] = b.y; r.v[6] = b.z; r.v[7] = b.w;
}
template <class M>
__device__ __forceinline__ void fload_nc(Fe<M>& r, const void* p) {
    const uint4* q = reinterpret_cast<const uint4*>(p);
    uint4 a = __ldg(q), b = __ldg(q + 1);
    r.v[0] = a.x; r.v[1] = a.y; r.v[2] = a.z; r.v[3] = a.w;
    r.v[4] = b.x; r.v[5] = b.y; r.v[6] = b.z; r.v[7] = b.w;
}
template <class M>
__device__ __forceinline__ void fstore(void* p, const Fe<M>& a) {
    uint4* q = reinterpret_cast<uint4*>(p);
    q[0] = make_uint4(a.v[0], a.v[1], a.v[2], a.v[3]);
    q[1] = make_uint4(a.v[4], a.v[5], a.v[6], a.v[7]);
}
__device__ __forceinline__ void fload(Fp2& r, const void* p) {
    fload(r.c0, p);
    fload(r.c1, reinterpret_cast<const char*>(p) + 32);
}
__device__ __forceinline__ void fload_nc(Fp2& r, const void* p) {
    fload_nc(r.c0, p);
    fload_nc(r.c1, reinterpret_cast<const char*>(p) + 32);
}
__device__ __forceinline__ void fstore(void* p, const Fp2& a) {
    fstore(p, a.c0);
    fstore(reinterpret_cast<char*>(p) + 32, a.c1);
}

__device__ __forceinline__ void fmulsub(Fp2& r, const Fp2& a, const Fp2& b, const Fp2& c, const Fp2& d) {
    Fp2 x, y;
    fmul(x, a, b);
    fmul(y, c, d);
    fsub(r, x, y);
}

}  // namespace zk
