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

#include <algorithm>

namespace zk {

static constexpr int kBaRounds = 3;
static constexpr uint32_t kBaItems = 32;  // outputs per thread in passes A and B
static constexpr int kBaThreads = 128;
static constexpr int kTreeLeaves = 512;   // product-tree leaves per block (256 threads)

// r = a^(p - 2) = a^-1 (Fermat), a != 0; one thread
__device__ __noinline__ void fp_inv_fermat(Fp& r, const Fp& a) {
    Fp acc, base = a;
    fset_one(acc);
    for (int w = 7; w >= 0; w--) {
        uint32_t e = ModP::m(w) - (w == 0 ? 2u : 0u);  // p - 2 (p's low word exceeds 2)
        for (int b = 31; b >= 0; b--) {
            Fp t;
            fsqr(t, acc);
            acc = t;
            if ((e >> b) & 1) {
                fmul(t, acc, base);
                acc = t;
            }
        }
    }
    r = acc;
}

// ---------------------------------------------------------------- level offsets
// counts[g] = ceil(c_g / 2^k) with c_g = offsets[g + 1] - offsets[g]
__global__ void ba_level_counts_kernel(const uint32_t* __restrict__ offsets, uint32_t nb, int k, uint32_t* __restrict__ counts) {
    for (uint32_t g = blockIdx.x * blockDim.x + threadIdx.x; g < nb; g += gridDim.x * blockDim.x) {
        const uint32_t c = offsets[g + 1] - offsets[g];
        counts[g] = (c + (1u << k) - 1) >> k;
    }
}

// element i of a level: a key (level 0: point index and sign) or a stored point
template <bool kKeys>
__device__ __forceinline__ void ba_load(Affine<Fp>& a, bool& inf, const uint32_t* keys, const uint8_t* pts, uint32_t i, bool need_y) {
    const uint8_t* p;
    uint32_t neg = 0;
    if (kKeys) {
        const uint32_t key = keys[i];
        p = pts + (size_t)(key & 0x7fffffffu) * 64;
        neg = key >> 31;
    } else {
        p = pts + (size_t)i * 64;
    }
    fload_nc(a.x, p);
    if (need_y) {
        fload_nc(a.y, p + 32);
        inf = fis_zero(a.x) && fis_zero(a.y);
        if (neg && !inf) {
            Fp t;
            fneg(t, a.y);
            a.y = t;
        }
    } else {
        // x = 0 is not on the curve (0 + 3 is not a square mod p), so x alone tells infinity
        inf = fis_zero(a.x);
    }
}

// bucket of output position q: off_out[g] <= q < off_out[g + 1]
__device__ __forceinline__ uint32_t ba_find_bucket(const uint32_t* off, uint32_t nb, uint32_t q) {
    uint32_t lo = 0, hi = nb;
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (off[mid] <= q) lo = mid; else hi = mid;
    }
    return lo;
}

// Pass A: for each output position q of this thread (kBaItems consecutive),
// the pair (2j, 2j + 1) of its bucket's input elements; a regular pair
// contributes d = x2 - x1 to the thread's running product, whose value before
// d is kept in prefix[q].  totals[t] = the thread's product (one if none).
template <bool kKeys>
__global__ void __launch_bounds__(kBaThreads) ba_pass_a_kernel(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ off_in,
                                                              const uint8_t* __restrict__ pts_in, const uint32_t* __restrict__ off_out,
                                                              uint32_t nb, Fp* __restrict__ prefix, Fp* __restrict__ totals,
                                                              size_t nthreads, unsigned long long* __restrict__ pair_count) {
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nthreads) return;
    Fp acc;
    fset_one(acc);
    const uint32_t N = off_out[nb];
    const size_t q0 = t * kBaItems;
    uint32_t regular = 0;
    if (q0 < N) {
        const uint32_t q1 = (uint32_t)std::min<size_t>(q0 + kBaItems, N);
        uint32_t g = ba_find_bucket(off_out, nb, (uint32_t)q0);
        uint32_t g_end = off_out[g + 1];
        for (uint32_t q = (uint32_t)q0; q < q1; q++) {
            while (q >= g_end) { g++; g_end = off_out[g + 1]; }
            const uint32_t i0 = off_in[g] + 2 * (q - off_out[g]);
            if (i0 + 1 >= off_in[g + 1]) continue;  // the odd last element: copied in pass B
            Affine<Fp> a, b;
            bool ia, ib;
            ba_load<kKeys>(a, ia, keys, pts_in, i0, false);
            ba_load<kKeys>(b, ib, keys, pts_in, i0 + 1, false);
            if (ia || ib || feq(a.x, b.x)) continue;  // exceptional: resolved alone in pass B
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

// Pass B: the pairs of pass A backwards, 1/d_q = (running inverse) x prefix[q],
// then the running inverse times d_q; writes each output point (all-zero for
// the point at infinity).
template <bool kKeys>
__global__ void __launch_bounds__(kBaThreads) ba_pass_b_kernel(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ off_in,
                                                              const uint8_t* __restrict__ pts_in, const uint32_t* __restrict__ off_out,
                                                              uint32_t nb, const Fp* __restrict__ prefix, const Fp* __restrict__ inv_totals,
                                                              size_t nthreads, uint8_t* __restrict__ pts_out) {
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nthreads) return;
    const uint32_t N = off_out[nb];
    const size_t q0 = t * kBaItems;
    if (q0 >= N) return;
    const uint32_t q1 = (uint32_t)std::min<size_t>(q0 + kBaItems, N);
    Fp inv;
    fload(inv, inv_totals + t);
    uint32_t g = ba_find_bucket(off_out, nb, q1 - 1);
    uint32_t g_begin = off_out[g];
    for (uint32_t q = q1; q-- > (uint32_t)q0;) {
        while (q < g_begin) { g--; g_begin = off_out[g]; }
        const uint32_t i0 = off_in[g] + 2 * (q - g_begin);
        Affine<Fp> a, b, o;
        bool ia, ib;
        ba_load<kKeys>(a, ia, keys, pts_in, i0, true);
        const bool pair = i0 + 1 < off_in[g + 1];
        if (pair) {
            ba_load<kKeys>(b, ib, keys, pts_in, i0 + 1, true);
        } else {
            ib = true;
        }
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
            fp_inv_fermat(id, d2);
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
        fstore(pts_out + (size_t)q * 64, o.x);
        fstore(pts_out + (size_t)q * 64 + 32, o.y);
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
        fp_inv_fermat(r, v[0]);
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
