// msm_affine.cuh -- batch-affine rounds of the G1 bucket accumulation.
//
// The keys of a window are sorted by bucket; bucket g holds c_g points.  A
// round adds the points of every bucket in adjacent pairs, in affine
// coordinates: for P1 = (x1, y1), P2 = (x2, y2) with x1 != x2,
//   l = (y2 - y1) / (x2 - x1),  x3 = l^2 - x1 - x2,  y3 = l (x1 - x3) - y1,
// so that bucket g holds ceil(c_g / 2) points afterwards, stored densely in the
// next level's array (level offsets by an exclusive scan of ceil(c_g / 2^k)).
// All the divisions of a round share one field inversion (Montgomery's trick
// over the whole grid): pass A forms, per thread, the running product of its
// denominators (the prefix before each one is kept); a product tree over the
// per-thread totals is inverted at its root (one Fermat exponentiation) and
// pushed back down; pass B walks each thread's pairs backwards, recovering
// every 1/(x2 - x1) from the prefix and the running inverse.  Per addition:
// 5 products + 1 squaring (1480 IMAD on 8 x 32-bit limbs), against
// 8 products + 2 squarings (2320) for the mixed XYZZ addition of the serial
// accumulation.  After kBaRounds rounds the remaining points (about 1/8 of the
// keys plus one per bucket) are summed by the XYZZ accumulation, which handles
// any bucket size (the log-depth fixup over segments).
//
// Exceptional pairs (a point at infinity, x1 == x2) stay out of the shared
// product and are resolved in pass B: P + O = P, P + (-P) = O, and a doubling
// (P + P, a repeated point) with its own inversion.
#pragma once
#include "curve.cuh"

namespace zk {
__device__ __forceinline__ void store_point(uint8_t* p, const Affine<Fp>& a) {
    fstore(p, a.x);
    fstore(p + 32, a.y);
}
}  // namespace zk

#include <algorithm>

namespace zk {

static constexpr int kBaRounds = 3;
static constexpr uint32_t kBaItems = 32;  // outputs per thread in passes A and B
static constexpr int kBaThreads = 128;
static constexpr int kTreeLeaves = 512;   // product-tree leaves per block (256 threads)

// r = a^-1 for a != 0 (Montgomery in, Montgomery out): the binary extended
// Euclidean algorithm on the plain value of a R (variable time: the values
// inverted here are products of public point coordinates), giving (a R)^-1,
// then one Montgomery product with R^3 for a^-1 R.  About 4x faster than a
// Fermat exponentiation in the one thread that runs it.
__device__ __noinline__ void fp_inv(Fp& r, const Fp& a) {
    uint32_t u[8], v[8], x1[8], x2[8];
    uint32_t nz = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        u[k] = a.v[k];
        v[k] = ModP::m(k);
        x1[k] = k == 0;
        x2[k] = 0;
        nz |= a.v[k];
    }
    if (!nz) { fset_zero(r); return; }
    auto is_one = [](const uint32_t* w) {
        uint32_t o = w[0] ^ 1u;
#pragma unroll
        for (int k = 1; k < 8; k++) o |= w[k];
        return o == 0;
    };
    auto shr1 = [](uint32_t* w) {
#pragma unroll
        for (int k = 0; k < 7; k++) w[k] = __funnelshift_r(w[k], w[k + 1], 1);
        w[7] >>= 1;
    };
    auto add_p = [](uint32_t* w) {  // w + p < 2^255: no carry out
        uint64_t c = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            c += (uint64_t)w[k] + ModP::m(k);
            w[k] = (uint32_t)c;
            c >>= 32;
        }
    };
    auto half_mod = [&](uint32_t* w) {  // w / 2 mod p for w < p
        if (w[0] & 1) add_p(w);
        shr1(w);
    };
    auto geq = [](const uint32_t* a_, const uint32_t* b_) {
        for (int k = 7; k >= 0; k--)
            if (a_[k] != b_[k]) return a_[k] > b_[k];
        return true;
    };
    auto sub = [](uint32_t* a_, const uint32_t* b_) {  // a -= b, a >= b
        int64_t c = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            c += (int64_t)a_[k] - b_[k];
            a_[k] = (uint32_t)c;
            c >>= 32;
        }
    };
    auto sub_mod = [&](uint32_t* a_, const uint32_t* b_) {  // a = a - b mod p, both < p
        if (geq(a_, b_)) {
            sub(a_, b_);
        } else {
            add_p(a_);
            sub(a_, b_);
        }
    };
    // at most ~2 x 254 halvings and ~2 x 254 subtractions in all; every loop is
    // bounded (u or v can only reach zero for a non-invertible input, which
    // the caller never passes, and then the result is meaningless, not a hang)
    int steps = 0;
    for (int it = 0; it < 2048 && !is_one(u) && !is_one(v); it++) {
        while (!(u[0] & 1) && steps < 4096) { shr1(u); half_mod(x1); steps++; }
        while (!(v[0] & 1) && steps < 4096) { shr1(v); half_mod(x2); steps++; }
        if (geq(u, v)) {
            sub(u, v);
            sub_mod(x1, x2);
        } else {
            sub(v, u);
            sub_mod(x2, x1);
        }
    }
    Fp x, r2, r3;
    const uint32_t* res = is_one(u) ? x1 : x2;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        x.v[k] = res[k];
        r2.v[k] = ModP::r2(k);
    }
    fmul(r3, r2, r2);  // R^3 (Montgomery form of R^2)
    fmul(r, x, r3);    // (a R)^-1 R^3 R^-1 = a^-1 R
}

// ---------------------------------------------------------------- level offsets
// counts[g] = ceil(c_g / 2^k) with c_g = offsets[g + 1] - offsets[g]
__global__ void ba_level_counts_kernel(const uint32_t* __restrict__ offsets, uint32_t nb, int k, uint32_t* __restrict__ counts) {
    for (uint32_t g = blockIdx.x * blockDim.x + threadIdx.x; g < nb; g += gridDim.x * blockDim.x) {
        const uint32_t c = offsets[g + 1] - offsets[g];
        counts[g] = (c + (1u << k) - 1) >> k;
    }
}

// bucket of output position q: the last g with off[g] <= q
__device__ __forceinline__ uint32_t ba_find_bucket(const uint32_t* off, uint32_t nb, uint32_t q) {
    uint32_t lo = 0, hi = nb;
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (off[mid] <= q) lo = mid; else hi = mid;
    }
    return lo;
}

// A point of a level array (all-zero: infinity)
__device__ __forceinline__ void ba_load_point(Affine<Fp>& a, bool& inf, const uint8_t* pts, uint32_t i) {
    load_affine(a, pts + (size_t)i * 64);
    inf = fis_zero(a.x) && fis_zero(a.y);
}
// The point of a key (point index, sign) from the input points
__device__ __forceinline__ void ba_gather(Affine<Fp>& a, const uint32_t* keys, const uint8_t* points, uint32_t i) {
    const uint32_t key = keys[i];
    load_affine(a, points + (size_t)(key & 0x7fffffffu) * 64);
    if ((key >> 31) && !(fis_zero(a.x) && fis_zero(a.y))) {
        Fp t;
        fneg(t, a.y);
        a.y = t;
    }
}

// Work of a thread: kBaItems output positions of the next level, interleaved
// over the 32 lanes of its warp (lane l: base + l + 32 i), so that a warp's
// loads and stores of one step are contiguous.
__device__ __forceinline__ size_t ba_warp_base(size_t t) { return (t >> 5) * 32 * kBaItems + (t & 31); }

// Pass A: for each output position q of this thread, the pair (2j, 2j + 1) of
// its bucket's input elements; a regular pair contributes d = x2 - x1 to the
// thread's running product, whose value before d is kept in prefix[q];
// totals[t] = the thread's product (one if none).  kGather (the first round):
// the elements are gathered from the keys and points and written, signs
// applied, into the dense level-0 array `dense` in key order, so that every
// later pass reads contiguous memory; else they are read from pts_in.
template <bool kGather>
__global__ void __launch_bounds__(kBaThreads) ba_pass_a_kernel(const uint32_t* __restrict__ keys, const uint8_t* __restrict__ points,
                                                              uint8_t* __restrict__ dense, const uint32_t* __restrict__ off_in,
                                                              const uint8_t* __restrict__ pts_in, const uint32_t* __restrict__ off_out,
                                                              uint32_t nb, Fp* __restrict__ prefix, Fp* __restrict__ totals,
                                                              size_t nthreads, unsigned long long* __restrict__ pair_count) {
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nthreads) return;
    Fp acc;
    fset_one(acc);
    const uint32_t N = off_out[nb];
    const size_t qb = ba_warp_base(t);
    uint32_t regular = 0;
    if (qb < N) {
        uint32_t g = ba_find_bucket(off_out, nb, (uint32_t)qb);
        uint32_t g_end = off_out[g + 1];
        for (uint32_t i = 0; i < kBaItems; i++) {
            const size_t qs = qb + (size_t)32 * i;
            if (qs >= N) break;
            const uint32_t q = (uint32_t)qs;
            while (q >= g_end) { g++; g_end = off_out[g + 1]; }
            const uint32_t i0 = off_in[g] + 2 * (q - off_out[g]);
            const bool pair = i0 + 1 < off_in[g + 1];
            Affine<Fp> a, b;
            bool ia, ib = true;
            if (kGather) {
                ba_gather(a, keys, points, i0);
                store_point(dense + (size_t)i0 * 64, a);
                ia = fis_zero(a.x) && fis_zero(a.y);
                if (pair) {
                    ba_gather(b, keys, points, i0 + 1);
                    store_point(dense + (size_t)(i0 + 1) * 64, b);
                    ib = fis_zero(b.x) && fis_zero(b.y);
                }
            } else {
                // x = 0 is not on the curve (3 is not a square mod p): x alone tells infinity
                fload_nc(a.x, pts_in + (size_t)i0 * 64);
                ia = fis_zero(a.x);
                if (pair) {
                    fload_nc(b.x, pts_in + (size_t)(i0 + 1) * 64);
                    ib = fis_zero(b.x);
                }
            }
            if (ia || ib || feq(a.x, b.x)) continue;  // no pair or exceptional: resolved alone in pass B
            Fp d, nxt;
            fsub(d, b.x, a.x);
            fstore(prefix + q, acc);
            fmul(nxt, acc, d);
            acc = nxt;
            regular++;
        }
    }
    fstore(totals + t, acc);
    if (regular) atomicAdd(pair_count, (unsigned long long)regular);
}

// Pass B: this thread's pairs backwards, 1/d_q = (running inverse) x prefix[q],
// then the running inverse times d_q; writes each output point of the next
// level (all-zero for the point at infinity).
__global__ void __launch_bounds__(kBaThreads) ba_pass_b_kernel(const uint32_t* __restrict__ off_in, const uint8_t* __restrict__ pts_in,
                                                              const uint32_t* __restrict__ off_out, uint32_t nb,
                                                              const Fp* __restrict__ prefix, const Fp* __restrict__ inv_totals,
                                                              size_t nthreads, uint8_t* __restrict__ pts_out) {
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nthreads) return;
    const uint32_t N = off_out[nb];
    const size_t qb = ba_warp_base(t);
    if (qb >= N) return;
    const uint32_t last = (uint32_t)std::min<size_t>(kBaItems - 1, (N - 1 - qb) / 32);  // items 0 .. last have q < N
    Fp inv;
    fload(inv, inv_totals + t);
    uint32_t g = ba_find_bucket(off_out, nb, (uint32_t)(qb + (size_t)32 * last));
    uint32_t g_begin = off_out[g];
    for (int i = (int)last; i >= 0; i--) {
        const uint32_t q = (uint32_t)(qb + (size_t)32 * i);
        while (q < g_begin) { g--; g_begin = off_out[g]; }
        const uint32_t i0 = off_in[g] + 2 * (q - g_begin);
        Affine<Fp> a, b, o;
        bool ia, ib = true;
        ba_load_point(a, ia, pts_in, i0);
        if (i0 + 1 < off_in[g + 1]) ba_load_point(b, ib, pts_in, i0 + 1);
        if (ia && ib) {
            fset_zero(o.x);
            fset_zero(o.y);
        } else if (ib) {
            o = a;
        } else if (ia) {
            o = b;
        } else if (!feq(a.x, b.x)) {
            Fp d, id, l, t2;
            fsub(d, b.x, a.x);
            fload(t2, prefix + q);
            fmul(id, inv, t2);   // 1 / d
            fmul(t2, inv, d);    // the running inverse without d
            inv = t2;
            fsub(t2, b.y, a.y);
            fmul(l, t2, id);     // l = (y2 - y1) / (x2 - x1)
            fsqr(t2, l);
            fsub(t2, t2, a.x);
            fsub(o.x, t2, b.x);  // x3 = l^2 - x1 - x2
            fsub(t2, a.x, o.x);
            fmul(l, l, t2);
            fsub(o.y, l, a.y);   // y3 = l (x1 - x3) - y1
        } else if (feq(a.y, b.y)) {
            // P + P: l = 3 x^2 / (2 y) with an inversion of its own (a repeated point)
            Fp x2, n3, d2, id, l, t2;
            fsqr(x2, a.x);
            fadd(n3, x2, x2);
            fadd(n3, n3, x2);
            fadd(d2, a.y, a.y);
            fp_inv(id, d2);
            fmul(l, n3, id);
            fsqr(t2, l);
            fsub(t2, t2, a.x);
            fsub(o.x, t2, a.x);
            fsub(t2, a.x, o.x);
            fmul(l, l, t2);
            fsub(o.y, l, a.y);
        } else {  // P + (-P)
            fset_zero(o.x);
            fset_zero(o.y);
        }
        store_point(pts_out + (size_t)q * 64, o);
    }
}

// ---------------------------------------------------------------- batch inversion
// Product tree over n values in blocks of kTreeLeaves leaves (heap order:
// node 1 the block's product, nodes kTreeLeaves.. the leaves, padded with one).
__global__ void __launch_bounds__(256) bt_up_kernel(const Fp* __restrict__ vals, size_t n, Fp* __restrict__ nodes, Fp* __restrict__ roots) {
    __shared__ Fp heap[2 * kTreeLeaves];
    const size_t base = (size_t)blockIdx.x * kTreeLeaves;
    for (int i = threadIdx.x; i < kTreeLeaves; i += blockDim.x) {
        Fp v;
        if (base + i < n) fload(v, vals + base + i);
        else fset_one(v);
        heap[kTreeLeaves + i] = v;
    }
    __syncthreads();
    for (int size = kTreeLeaves / 2; size >= 1; size >>= 1) {
        for (int i = threadIdx.x; i < size; i += blockDim.x) {
            Fp p;
            fmul(p, heap[2 * (size + i)], heap[2 * (size + i) + 1]);
            heap[size + i] = p;
        }
        __syncthreads();
    }
    Fp* out = nodes + (size_t)blockIdx.x * 2 * kTreeLeaves;
    for (int i = threadIdx.x; i < 2 * kTreeLeaves; i += blockDim.x) out[i] = heap[i];
    if (threadIdx.x == 0) roots[blockIdx.x] = heap[1];
}

__global__ void bt_invert_kernel(Fp* v) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        Fp r;
        fp_inv(r, v[0]);
        v[0] = r;
    }
}

// inverses of a block's leaves from the inverse of its product (parent_inv[block]):
// top-down, each node's slot turns from its value into its inverse once its
// parent (whose thread reads both children before writing either) is done
__global__ void __launch_bounds__(256) bt_down_kernel(const Fp* __restrict__ nodes, const Fp* __restrict__ parent_inv, size_t n,
                                                      Fp* __restrict__ out_inv) {
    __shared__ Fp h[2 * kTreeLeaves];
    const Fp* in = nodes + (size_t)blockIdx.x * 2 * kTreeLeaves;
    for (int i = threadIdx.x; i < 2 * kTreeLeaves; i += blockDim.x) h[i] = in[i];
    __syncthreads();
    if (threadIdx.x == 0) h[1] = parent_inv[blockIdx.x];
    __syncthreads();
    for (int size = 1; size < kTreeLeaves; size <<= 1) {
        for (int i = threadIdx.x; i < size; i += blockDim.x) {
            const int node = size + i;
            const Fp l = h[2 * node], r = h[2 * node + 1], iv = h[node];
            Fp a, b;
            fmul(a, iv, r);  // 1/left = 1/node x right
            fmul(b, iv, l);  // 1/right = 1/node x left
            h[2 * node] = a;
            h[2 * node + 1] = b;
        }
        __syncthreads();
    }
    const size_t base = (size_t)blockIdx.x * kTreeLeaves;
    for (int i = threadIdx.x; i < kTreeLeaves; i += blockDim.x)
        if (base + i < n) fstore(out_inv + base + i, h[kTreeLeaves + i]);
}

}  // namespace zk
