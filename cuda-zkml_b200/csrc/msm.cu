// msm.cu -- Pippenger multi-scalar multiplication over BN254 G1 and G2 on
// sm_100a.
//
// Replaces the reference's msm_g1 / msm_g2 (src/msm/msm.cu:320-442, :526-598),
// which accumulate with one global spin lock per bucket and reduce each window
// on a single thread.  This pipeline has no locks and no unbounded waits:
//
//   1. count    : per scalar, Montgomery -> standard form, signed c-bit digits
//                 d in [-2^(c-1), 2^(c-1)] (Booth-style recoding, so a window
//                 has 2^(c-1) buckets instead of the reference's 2^c - 1), and
//                 a histogram of (window, |d|) over all nonzero digits.
//   2. scan     : exclusive prefix sum of the histogram -> bucket offsets.
//   3. scatter  : counting sort; key = sign << 31 | point index, grouped by
//                 (window, bucket).  All windows share one flat key array.
//   4. accumulate: the flat key array is cut into equal segments, one thread
//                 each, so the work per thread is fixed however skewed the
//                 scalars are.  A thread sums its keys' points run by run into
//                 XYZZ accumulators (mixed additions, points gathered with
//                 128-bit loads); a run that covers a whole bucket is written
//                 straight to the bucket, a run cut by a segment boundary goes
//                 to one of two per-thread partial slots.
//   5. fixup    : buckets that straddle segments sum their partial slots.
//   6. reduce   : per window, chunks of buckets are reduced in parallel with
//                 the running-sum identity sum_b (b+1) S_b (msm.cu:298-304),
//                 each chunk corrected by lo * (chunk sum) with a short
//                 double-and-add.
//   7. windows  : one block per window tree-sums the chunk results.
//   8. combine  : the W window sums go to the host, which does the Horner
//                 combine sum_w 2^(c w) S_w (msm.cu:423-430) and the affine
//                 normalisation.
#include "curve.cuh"
#include "host_field.hpp"
#include "msm_affine.cuh"
#include "runtime.cuh"

#include <algorithm>
#include <cstring>
#include <type_traits>
#include <vector>

namespace zk {

// ------------------------------------------------------------------ plan
struct MsmPlan {
    int c = 0;           // window bits
    int W = 0;           // windows, W * c >= 255 so the top carry is absorbed
    uint32_t B = 0;      // buckets per window = 2^(c-1)
    uint32_t nb = 0;     // W * B
    uint32_t seg = 0;    // keys per accumulate thread
    size_t max_keys = 0; // n * W
    size_t max_segs = 0;
    uint32_t chunk = 0;  // buckets per reduce thread
    uint32_t tw = 0;     // reduce threads per window
    uint32_t chunk2 = 0; // chunk results per second-level thread
    uint32_t tw2 = 0;    // second-level threads per window
    uint32_t tiles = 0;  // scan tiles
    bool agg = false;    // warp-aggregated bucket atomics (many equal digits)
    // window w's digits go to buckets w * wstride + b and keys i + w * kstride:
    // (B, 0) for W separate windows; (0, n) for precomputed window tables,
    // where the point of (i, w) is 2^(c w) P_i, stored at index i + w n
    uint32_t wstride = 0;
    size_t kstride = 0;
    // batch-affine rounds before the XYZZ accumulation (msm_affine.cuh): 0 or
    // kBaRounds; bound of the elements left after them, and the accumulation's
    // segment length over those
    int ba = 0;
    size_t ba_left = 0;
    uint32_t ba_seg = 0;
    size_t key_bound = 0;
};

static constexpr int kScanTile = 4096;  // 1024 threads x 4

// Window width c minimising the Fp multiplications of the whole MSM: one mixed
// addition (10 mul) per nonzero signed digit, plus 2^(c-1) running-sum steps
// (2 full additions, 14 mul each, plus the chunk correction) for every window
// that holds digits.  `hist[b]` counts scalars of bit length b; a b-bit scalar
// has at most ceil((b + 1) / c) nonzero digits.  Without a histogram every
// scalar counts as 254 bits.  ZK_MSM_WINDOW_BITS / ZK_MSM_G2_WINDOW_BITS
// override the choice.
static int choose_window_bits(size_t n, bool g2, const uint32_t* hist) {
    const char* env = getenv(g2 ? "ZK_MSM_G2_WINDOW_BITS" : "ZK_MSM_WINDOW_BITS");
    if (env && atoi(env) >= 2 && atoi(env) <= 22) return atoi(env);
    int maxbits = 254;
    if (hist) {
        maxbits = 0;
        for (int b = 0; b < 256; b++)
            if (hist[b]) maxbits = b;
    }
    int best = 3;
    double best_cost = 1e300;
    for (int c = 3; c <= (g2 ? 18 : 21); c++) {
        double digits = 0;
        if (hist) {
            for (int b = 1; b < 256; b++) digits += (double)hist[b] * (double)((b + 1 + c - 1) / c);
        } else {
            digits = (double)n * ((255 + c - 1) / c);
        }
        const double windows = (maxbits + 1 + c - 1) / c;
        const double cost = digits * 10.0 + windows * (double)(1u << (c - 1)) * 30.0;
        if (cost < best_cost) { best_cost = cost; best = c; }
    }
    return best;
}

static uint32_t pow2_clamp(double x, uint32_t lo, uint32_t hi) {
    uint32_t p = lo;
    while (p < hi && (double)p * 2 <= x) p *= 2;
    return p;
}

// Upper bound on the keys (nonzero signed digits): a b-bit scalar has at most
// ceil((b + 1) / c) of them.
static size_t plan_key_bound(const MsmPlan& p, const uint32_t* hist) {
    size_t key_bound = p.max_keys;
    if (hist) {
        size_t d = 0;
        for (int b = 1; b < 256; b++) d += (size_t)hist[b] * (size_t)((b + 1 + p.c - 1) / p.c);
        key_bound = std::min(key_bound, d);
    }
    return key_bound;
}

// hist_exact: `hist` counts every scalar of the MSM (not an estimate from a
// sample), so the windows above the longest scalar's top digit hold no digit
// and are left out.
static MsmPlan make_plan(size_t n, bool g2, const uint32_t* hist, int num_sms, bool hist_exact = true) {
    MsmPlan p;
    p.c = choose_window_bits(n, g2, hist);
    p.W = (255 + p.c - 1) / p.c;
    if (hist && hist_exact) {
        int maxbits = 0;
        for (int b = 0; b < 256; b++)
            if (hist[b]) maxbits = b;
        // a b-bit scalar's signed digits fill ceil((b + 1) / c) windows at most
        p.W = std::max(1, std::min(p.W, (maxbits + 1 + p.c - 1) / p.c));
    }
    p.B = 1u << (p.c - 1);
    p.nb = (uint32_t)p.W * p.B;
    p.max_keys = n * (size_t)p.W;
    const size_t key_bound = plan_key_bound(p, hist);
    // Keys per accumulate thread and buckets per reduce thread: long serial
    // chains when there is work for every SM many times over, short ones when
    // there is little (a witness MSM, a shard of one), so that enough threads
    // run to hide the latency of the dependent multiplications.
    const double sms = (double)std::max(num_sms, 1);
    p.seg = pow2_clamp((double)key_bound / (sms * 512.0), g2 ? 8 : 16, g2 ? 64 : 128);
    p.max_segs = std::max<size_t>(1, (key_bound + p.seg - 1) / p.seg);
    p.chunk = std::min<uint32_t>(p.B, pow2_clamp((double)p.nb / (sms * 256.0), 2, 32));
    p.tw = p.B / p.chunk;
    p.chunk2 = std::min<uint32_t>(p.tw, pow2_clamp((double)p.W * p.tw / (sms * 64.0), 2, 16));
    p.tw2 = p.tw / p.chunk2;
    p.tiles = (p.nb + 1 + kScanTile - 1) / kScanTile;
    // Scalars 1..3 (0/1 range-check bits of a witness) all fall in window 0's
    // first buckets: one atomic per warp and bucket instead of one per lane.
    // For spread-out scalars the grouping costs more than it saves.
    p.agg = hist && ((size_t)hist[1] + hist[2]) * 256 >= n;
    p.wstride = p.B;
    p.kstride = 0;
    return p;
}

// The counting sort counts, offsets and indexes keys in 32 bits (bucket
// offsets, segment starts, sign << 31 | point index), so a pass may hold at
// most 2^31 - 1 keys.  With the widest window the cost model picks for
// full-width scalars (c = 21, W = 13) kMaxPassPoints points give 1.74e9 keys;
// larger MSMs run in passes of at most that many points.
static constexpr size_t kMaxKeys = 0x7fffffffull;
static constexpr size_t kMaxPassPoints = (size_t)1 << 27;

// A window width forced by ZK_MSM_WINDOW_BITS fixes W, and with it the worst
// case n W, before any device work: refuse a pass that cannot fit.
static int check_forced_window(size_t n, bool g2) {
    const char* env = getenv(g2 ? "ZK_MSM_G2_WINDOW_BITS" : "ZK_MSM_WINDOW_BITS");
    if (!env || atoi(env) < 2 || atoi(env) > 22) return ZK_OK;
    const int c = atoi(env);
    const size_t W = (255 + c - 1) / c;
    if (n * W > kMaxKeys) {
        set_error("msm: %zu points with the forced window width %d (%zu windows) exceed 2^31 - 1 keys", n, c, W);
        return ZK_ERR_RANGE;
    }
    return ZK_OK;
}

// The plan's proven key bound (from the scalars' bit lengths) must fit too.
static int check_key_bound(const MsmPlan& p, const uint32_t* hist) {
    const size_t bound = plan_key_bound(p, hist);
    if (bound > kMaxKeys) {
        set_error("msm: up to %zu keys with window width %d exceed 2^31 - 1", bound, p.c);
        return ZK_ERR_RANGE;
    }
    return ZK_OK;
}

// ------------------------------------------------------------------ digits
// Signed-digit recoding of a standard-form scalar held in v[0..7], consumed
// c bits at a time from the bottom (the 256-bit value is shifted in place).
__device__ __forceinline__ int next_digit(uint32_t v[8], int c, uint32_t& carry) {
    uint32_t raw = (v[0] & ((1u << c) - 1)) + carry;
#pragma unroll
    for (int i = 0; i < 7; i++) v[i] = __funnelshift_r(v[i], v[i + 1], c);
    v[7] >>= c;
    uint32_t half = 1u << (c - 1);
    if (raw > half) {
        carry = 1;
        return (int)raw - (int)(1u << c);
    }
    carry = 0;
    return (int)raw;
}

// A standard-form scalar s above (r - 1) / 2 is replaced by r - s, and the
// caller negates its digits: s P = (r - s)(-P), the same point, so the result
// does not change.  A signed value -v of a zkML witness (stored as r - v) then
// costs the digits of v instead of a full-width scalar's; folded scalars have
// at most 253 bits.  Returns whether s was replaced.
__device__ __forceinline__ bool fold_scalar(uint32_t v[8]) {
    bool gt = false, decided = false;
#pragma unroll
    for (int k = 7; k >= 0; k--) {
        const uint32_t h = (ModR::m(k) >> 1) | (k < 7 ? ModR::m(k + 1) << 31 : 0u);  // (r - 1) / 2, r odd
        if (!decided && v[k] != h) {
            gt = v[k] > h;
            decided = true;
        }
    }
    if (gt) {
        uint32_t borrow = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const uint64_t d = (uint64_t)ModR::m(k) - v[k] - borrow;
            v[k] = (uint32_t)d;
            borrow = (uint32_t)(d >> 63);
        }
    }
    return gt;
}

// Bit lengths of the folded standard-form scalars (0..253), for the window choice.
__global__ void __launch_bounds__(256) msm_bitlen_hist_kernel(const Fr* __restrict__ scalars, size_t n, uint32_t* __restrict__ hist) {
    __shared__ uint32_t h[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) h[i] = 0;
    __syncthreads();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        Fr s;
        fload_nc(s, scalars + i);
        ffrom_mont(s, s);
        fold_scalar(s.v);
        int len = 0;
#pragma unroll
        for (int k = 7; k >= 0; k--)
            if (len == 0 && s.v[k]) len = 32 * k + 32 - __clz(s.v[k]);
        // uniform scalars put nearly every lane on the same length or two: one
        // shared-memory atomic per distinct length in the warp
        const unsigned peers = __match_any_sync(__activemask(), len);
        if ((threadIdx.x & 31) == (unsigned)(__ffs(peers) - 1)) atomicAdd(&h[len], (uint32_t)__popc(peers));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += blockDim.x)
        if (h[i]) atomicAdd(&hist[i], h[i]);
}

// Digits are stored window-major (digits[w * n + i] = sign << 31 | bucket + 1,
// 0 for a zero digit) so that the scatter can run one window after another.
// The lanes of a warp that hit the same bucket add their count with one atomic
// (witness scalars put most digits in one bucket: 0/1 range-check bits).
// Scalars are folded (fold_scalar): the digits of r - s with their signs flipped.
template <bool kAgg>
__global__ void msm_count_kernel(const Fr* __restrict__ scalars, size_t n, int c, int W, uint32_t wstride,
                                 uint32_t* __restrict__ counts, uint32_t* __restrict__ digits) {
    const uint32_t lane = threadIdx.x & 31;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        Fr s;
        fload_nc(s, scalars + i);
        ffrom_mont(s, s);
        const bool neg = fold_scalar(s.v);
        uint32_t carry = 0;
        for (int w = 0; w < W; w++) {
            const int d = next_digit(s.v, c, carry);
            uint32_t code = 0, key = 0xffffffffu;
            if (d) {
                const uint32_t b = (uint32_t)(d < 0 ? -d : d) - 1;
                key = (uint32_t)w * wstride + b;
                code = ((d < 0) != neg ? 0x80000000u : 0u) | (b + 1);
            }
            if (kAgg) {
                const uint32_t peers = __match_any_sync(__activemask(), key);
                if (d && lane == (uint32_t)(__ffs(peers) - 1)) atomicAdd(&counts[key], (uint32_t)__popc(peers));
            } else if (d) {
                atomicAdd(&counts[key], 1u);
            }
            digits[(size_t)w * n + i] = code;
        }
    }
}

// Counting-sort scatter, window-major: block b covers window b / blocks_per_window,
// so the blocks resident at any time touch one window's cursors (2^(c-1) words)
// and key range (about n words), which stay in L2; scattering all windows at once
// wrote partial sectors all over the whole key array.
template <bool kAgg>
__global__ void __launch_bounds__(256) msm_scatter_kernel(const uint32_t* __restrict__ digits, size_t n, uint32_t wstride,
                                                          size_t kstride, uint32_t blocks_per_window, uint32_t* __restrict__ cursors,
                                                          uint32_t* __restrict__ keys) {
    const uint32_t w = blockIdx.x / blocks_per_window;
    const size_t i = (size_t)(blockIdx.x % blocks_per_window) * blockDim.x + threadIdx.x;
    const uint32_t code = i < n ? digits[(size_t)w * n + i] : 0u;
    const uint32_t key = code ? w * wstride + (code & 0x7fffffffu) - 1 : 0xffffffffu;
    const uint32_t idx = (uint32_t)(i + w * kstride);  // < 2^31, checked by the caller
    if (!kAgg) {
        if (!code) return;
        keys[atomicAdd(&cursors[key], 1u)] = (code & 0x80000000u) | idx;
        return;
    }
    // lanes with the same bucket take consecutive slots from one atomic
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t peers = __match_any_sync(0xffffffffu, key);
    if (!code) return;
    const uint32_t leader = (uint32_t)(__ffs(peers) - 1);
    uint32_t base = 0;
    if (lane == leader) base = atomicAdd(&cursors[key], (uint32_t)__popc(peers));
    base = __shfl_sync(peers, base, leader);
    keys[base + (uint32_t)__popc(peers & ((1u << lane) - 1))] = (code & 0x80000000u) | idx;
}

// ------------------------------------------------------------------ scan
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t x, uint32_t* warp_sums, uint32_t& total) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint32_t incl = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sums[wid] = incl;
    __syncthreads();
    if (wid == 0) {
        uint32_t ws = lane < nw ? warp_sums[lane] : 0;
        uint32_t wi = ws;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t y = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += y;
        }
        if (lane < nw) warp_sums[lane] = wi - ws;
        if (lane == 31) warp_sums[32] = wi;
    }
    __syncthreads();
    uint32_t r = incl - x + warp_sums[wid];
    total = warp_sums[32];
    __syncthreads();
    return r;
}

// tile sums of counts[0..len)
__global__ void scan_tile_sums_kernel(const uint32_t* __restrict__ in, uint32_t len, uint32_t* __restrict__ tile_sums) {
    __shared__ uint32_t ws[33];
    uint32_t base = blockIdx.x * kScanTile + threadIdx.x * 4;
    uint32_t s = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) s += (base + k < len) ? in[base + k] : 0u;
    uint32_t total;
    block_exclusive_scan(s, ws, total);
    if (threadIdx.x == 0) tile_sums[blockIdx.x] = total;
}

// exclusive scan of the tile sums in place (single block)
__global__ void scan_tiles_kernel(uint32_t* __restrict__ tile_sums, uint32_t tiles) {
    __shared__ uint32_t ws[33];
    uint32_t carry = 0;
    for (uint32_t base = 0; base < tiles; base += blockDim.x) {
        uint32_t i = base + threadIdx.x;
        uint32_t x = i < tiles ? tile_sums[i] : 0u;
        uint32_t total;
        uint32_t ex = block_exclusive_scan(x, ws, total);
        if (i < tiles) tile_sums[i] = ex + carry;
        carry += total;
    }
}

// offsets[i] = exclusive prefix of counts, for i in [0, len]; cursors = copy
__global__ void scan_finish_kernel(const uint32_t* __restrict__ in, uint32_t len, const uint32_t* __restrict__ tile_offs,
                                   uint32_t* __restrict__ offsets, uint32_t* __restrict__ cursors) {
    __shared__ uint32_t ws[33];
    uint32_t base = blockIdx.x * kScanTile + threadIdx.x * 4;
    uint32_t v[4], s = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        v[k] = (base + k < len) ? in[base + k] : 0u;
        s += v[k];
    }
    uint32_t total;
    uint32_t ex = block_exclusive_scan(s, ws, total) + tile_offs[blockIdx.x];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        if (base + k <= len) {
            offsets[base + k] = ex;
            if (base + k < len) cursors[base + k] = ex;
        }
        ex += v[k];
    }
}

// ------------------------------------------------------------------ accumulate
// The point of a key: keys whose index lies outside [idx_lo, idx_hi) are skipped
// (an MSM over a sub-range of scalars that shares another MSM's sort); the
// others read point idx - idx_lo.
template <class Cv>
__device__ __forceinline__ void load_signed_point(Affine<typename Cv::F>& a, bool& is_inf, const uint8_t* points, uint32_t key,
                                                  uint32_t idx_lo, uint32_t idx_hi) {
    using F = typename Cv::F;
    uint32_t idx = key & 0x7fffffffu;
    if (idx < idx_lo || idx >= idx_hi) {
        is_inf = true;
        return;
    }
    load_affine(a, points + (size_t)(idx - idx_lo) * Cv::kAffineBytes);
    is_inf = fis_zero(a.x) && fis_zero(a.y);
    if (key >> 31) { F t; fneg(t, a.y); a.y = t; }
}

// kDirect: element p of a bucket is the point stored at position p (the level
// left by the batch-affine rounds: no key, no sign, all-zero = infinity).
template <class Cv, bool kDirect = false>
__global__ void __launch_bounds__(128, Cv::kAccumulateMinBlocks) msm_accumulate_kernel(
    const uint32_t* __restrict__ keys, const uint32_t* __restrict__ offsets, uint32_t nb, const uint8_t* __restrict__ points,
    uint32_t seg, uint8_t* __restrict__ bucket_sums, uint8_t* __restrict__ part_first, uint8_t* __restrict__ part_last,
    uint32_t* __restrict__ first_bucket, uint32_t* __restrict__ last_bucket, uint32_t idx_lo, uint32_t idx_hi,
    uint32_t* __restrict__ max_span) {
    using F = typename Cv::F;
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t K = offsets[nb];
    const size_t start = t * seg;
    if (start >= K) return;
    const uint32_t s0 = (uint32_t)start;
    const uint32_t s1 = (uint32_t)std::min<size_t>(start + seg, K);
    // bucket g with offsets[g] <= s0 < offsets[g+1]
    uint32_t lo = 0, hi = nb;
    while (hi - lo > 1) {
        uint32_t mid = (lo + hi) >> 1;
        if (offsets[mid] <= s0) lo = mid; else hi = mid;
    }
    uint32_t g = lo, g_begin = offsets[g], g_end = offsets[g + 1];
    uint32_t run_start = s0;
    Xyzz<F> acc;
    set_identity(acc);
    // A run covering its whole bucket goes straight to the bucket; a run cut by
    // the segment boundary goes to the "first" slot when it starts the segment,
    // else to the "last" slot (it then runs to the segment's end).
    auto flush = [&]() {
        uint8_t* dst;
        if (g_begin >= s0 && g_end <= s1) {
            dst = bucket_sums + (size_t)g * Cv::kXyzzBytes;
        } else {
            if (run_start == s0) {
                dst = part_first + t * Cv::kXyzzBytes;
                first_bucket[t] = g;
            } else {
                dst = part_last + t * Cv::kXyzzBytes;
                last_bucket[t] = g;
            }
            // the widest cut bucket bounds the fixup rounds that have work
            atomicMax(max_span, (g_end - 1) / seg - g_begin / seg + 1);
        }
        store_xyzz(dst, acc);
    };
    for (uint32_t p = s0; p < s1; p++) {
        if (p >= g_end) {
            flush();
            do { g++; g_end = offsets[g + 1]; } while (p >= g_end);
            g_begin = offsets[g];
            run_start = p;
            set_identity(acc);
        }
        Affine<F> a;
        bool inf;
        if (kDirect) {
            load_affine(a, points + (size_t)p * Cv::kAffineBytes);
            inf = fis_zero(a.x) && fis_zero(a.y);
        } else {
            load_signed_point<Cv>(a, inf, points, keys[p], idx_lo, idx_hi);
        }
        if (!inf) madd(acc, a);
    }
    flush();
}

// Buckets cut by segment boundaries.  Bucket g with keys [b0, b1) spans the
// segments sa = b0 / seg .. sb = (b1 - 1) / seg; its m = sb - sa + 1 partial
// sums are V_0 (slot "first" of sa when b0 starts that segment, else its
// "last" slot) and V_j = "first" slot of sa + j.  Round r of a binary tree adds
// V_{j + 2^r} into V_j for every j divisible by 2^(r + 1), so even a bucket
// holding millions of keys (the top window, or the many 0/1 scalars of a real
// witness) is summed in log2(m) parallel steps instead of m serial adds.  (A
// wider tree needs fewer launches but puts radix - 1 dependent additions in
// each round; on deep trees that measured slower.)
template <class Cv>
__global__ void msm_fixup_round_kernel(const uint32_t* __restrict__ offsets, const uint32_t* __restrict__ first_bucket,
                                       const uint32_t* __restrict__ last_bucket, size_t nseg, uint32_t seg, uint32_t stride,
                                       uint8_t* __restrict__ part_first, uint8_t* __restrict__ part_last,
                                       const uint32_t* __restrict__ max_span) {
    using F = typename Cv::F;
    if (stride >= *max_span) return;  // no bucket spans more than `stride` segments
    for (size_t s = (size_t)blockIdx.x * blockDim.x + threadIdx.x; s < nseg; s += (size_t)gridDim.x * blockDim.x) {
        const uint32_t gf = first_bucket[s], gl = last_bucket[s];
        if (gf != 0xffffffffu) {
            const uint32_t sa = offsets[gf] / seg, sb = (offsets[gf + 1] - 1) / seg;
            const uint32_t j = (uint32_t)s - sa, m = sb - sa + 1;
            if ((j & (2 * stride - 1)) == 0 && j + stride < m) {
                Xyzz<F> a, b;
                load_xyzz(a, part_first + s * Cv::kXyzzBytes);
                load_xyzz(b, part_first + (s + stride) * Cv::kXyzzBytes);
                add(a, b);
                store_xyzz(part_first + s * Cv::kXyzzBytes, a);
            }
        }
        if (gl != 0xffffffffu) {  // a "last" slot always holds V_0 of its bucket (sa = s)
            const uint32_t m = (offsets[gl + 1] - 1) / seg - (uint32_t)s + 1;
            if (stride < m) {
                Xyzz<F> a, b;
                load_xyzz(a, part_last + s * Cv::kXyzzBytes);
                load_xyzz(b, part_first + (s + stride) * Cv::kXyzzBytes);
                add(a, b);
                store_xyzz(part_last + s * Cv::kXyzzBytes, a);
            }
        }
    }
}

// after the rounds: V_0 of every cut bucket is its sum
template <class Cv>
__global__ void msm_fixup_final_kernel(const uint32_t* __restrict__ offsets, uint32_t nb, uint32_t seg, const uint8_t* __restrict__ part_first,
                                       const uint8_t* __restrict__ part_last, uint8_t* __restrict__ bucket_sums) {
    const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= nb) return;
    const uint32_t b0 = offsets[g], b1 = offsets[g + 1];
    if (b0 == b1) return;
    const uint32_t sa = b0 / seg, sb = (b1 - 1) / seg;
    if (sa == sb) return;  // whole bucket inside one segment: already written
    const uint8_t* src = (b0 == sa * seg ? part_first : part_last) + (size_t)sa * Cv::kXyzzBytes;
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(bucket_sums + (size_t)g * Cv::kXyzzBytes);
#pragma unroll
    for (int i = 0; i < Cv::kXyzzBytes / 16; i++) d4[i] = s4[i];
}

// ------------------------------------------------------------------ reduce
// The window sum is T_w = sum_b (b + 1) S_b over the bucket sums S_b.  Level 1:
// thread (w, j) takes the buckets [lo, lo + chunk), lo = j chunk, and forms
//   acc_j = sum (b - lo + 1) S_b   and   run_j = sum S_b
// by running sums, so that T_w = sum_j acc_j + chunk * U, U = sum_j j run_j.
// Level 2 forms U the same way over groups of chunk2 chunk results; only its
// few threads pay a double-and-add for their group's start, and the window
// kernel adds the pieces (chunk is a power of two: U is doubled log2(chunk)
// times).  One level with a double-and-add per chunk did ~30% more additions.
template <class Cv>
__global__ void msm_reduce_kernel(const uint32_t* __restrict__ offsets, const uint8_t* __restrict__ bucket_sums, int W, uint32_t B,
                                  uint32_t chunk, uint32_t tw, uint8_t* __restrict__ chunk_acc, uint8_t* __restrict__ chunk_run) {
    using F = typename Cv::F;
    uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    if (tid >= (uint32_t)W * tw) return;
    uint32_t w = tid / tw, j = tid % tw;
    uint32_t lo = j * chunk;
    Xyzz<F> run, acc, q;
    set_identity(run);
    set_identity(acc);
    for (uint32_t b = lo + chunk; b-- > lo;) {
        uint32_t g = w * B + b;
        if (!offsets || offsets[g] != offsets[g + 1]) {  // null: every bucket is written (the identity when empty)
            load_xyzz(q, bucket_sums + (size_t)g * Cv::kXyzzBytes);
            add(run, q);
        }
        add(acc, run);
    }
    store_xyzz(chunk_acc + (size_t)tid * Cv::kXyzzBytes, acc);
    store_xyzz(chunk_run + (size_t)tid * Cv::kXyzzBytes, run);
}

// thread (w, k): chunk results [k chunk2, (k + 1) chunk2) of window w ->
//   x_k = sum acc_j   and   u_k = sum_j j run_j
template <class Cv>
__global__ void msm_reduce2_kernel(const uint8_t* __restrict__ chunk_acc, const uint8_t* __restrict__ chunk_run, int W, uint32_t tw,
                                   uint32_t chunk2, uint32_t tw2, uint8_t* __restrict__ part_x, uint8_t* __restrict__ part_u) {
    using F = typename Cv::F;
    uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    if (tid >= (uint32_t)W * tw2) return;
    uint32_t w = tid / tw2, k = tid % tw2;
    uint32_t lo = k * chunk2;
    Xyzz<F> x, run, y, q;
    set_identity(x);
    set_identity(run);
    set_identity(y);
    for (uint32_t j = lo + chunk2; j-- > lo;) {
        const size_t r = (size_t)w * tw + j;
        add(y, run);  // before adding run_j: y = sum (j - lo) run_j
        load_xyzz(q, chunk_run + r * Cv::kXyzzBytes);
        add(run, q);
        load_xyzz(q, chunk_acc + r * Cv::kXyzzBytes);
        add(x, q);
    }
    // u_k = y + lo run
    if (lo && !is_identity(run)) {
        Xyzz<F> m;
        set_identity(m);
        int top = 31 - __clz(lo);
        for (int bit = top; bit >= 0; bit--) {
            Xyzz<F> d;
            dbl(d, m);
            m = d;
            if ((lo >> bit) & 1) add(m, run);
        }
        add(y, m);
    }
    store_xyzz(part_x + (size_t)tid * Cv::kXyzzBytes, x);
    store_xyzz(part_u + (size_t)tid * Cv::kXyzzBytes, y);
}

// Windows with many group results (one window over 2^19 buckets: the H MSM over
// precomputed tables): block (w, b, y) sums kWinPre consecutive x_k (y = 0) or
// u_k (y = 1) of window w into one entry, a tree over its threads, so that the
// one block per window that follows adds a few entries instead of thousands in
// a dependent chain (1.65 -> ~0.3 ms for 8192 entries).
static constexpr uint32_t kWinPre = 512;

template <class Cv>
__global__ void __launch_bounds__(256) msm_window_pre_kernel(const uint8_t* __restrict__ part_x, const uint8_t* __restrict__ part_u,
                                                             uint32_t tw2, uint32_t bpw, uint8_t* __restrict__ scratch,
                                                             uint8_t* __restrict__ out_x, uint8_t* __restrict__ out_u) {
    using F = typename Cv::F;
    const uint32_t w = blockIdx.x / bpw, b = blockIdx.x % bpw;
    const uint8_t* src = (blockIdx.y == 0 ? part_x : part_u) + (size_t)w * tw2 * Cv::kXyzzBytes;
    uint8_t* t = scratch + ((size_t)blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x * Cv::kXyzzBytes;
    Xyzz<F> acc, q;
    set_identity(acc);
    const uint32_t lo = b * kWinPre, hi = min(lo + kWinPre, tw2);
    for (uint32_t k = lo + threadIdx.x; k < hi; k += blockDim.x) {
        load_xyzz(q, src + (size_t)k * Cv::kXyzzBytes);
        add(acc, q);
    }
    store_xyzz(t + (size_t)threadIdx.x * Cv::kXyzzBytes, acc);
    __syncthreads();
    for (uint32_t s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            load_xyzz(acc, t + (size_t)threadIdx.x * Cv::kXyzzBytes);
            load_xyzz(q, t + (size_t)(threadIdx.x + s) * Cv::kXyzzBytes);
            add(acc, q);
            store_xyzz(t + (size_t)threadIdx.x * Cv::kXyzzBytes, acc);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        load_xyzz(acc, t);
        store_xyzz((blockIdx.y == 0 ? out_x : out_u) + (size_t)blockIdx.x * Cv::kXyzzBytes, acc);
    }
}

// one block per window: tree sums of the x_k and of the u_k, then
// T_w = sum x_k + chunk * sum u_k
template <class Cv>
constexpr int win_threads() { return std::is_same<Cv, G2>::value ? 128 : 256; }

template <class Cv>
__global__ void __launch_bounds__(win_threads<Cv>()) msm_window_kernel(const uint8_t* __restrict__ part_x, const uint8_t* __restrict__ part_u,
                                                                       uint32_t tw2, int log_chunk, uint8_t* __restrict__ scratch,
                                                                       uint8_t* __restrict__ window_sums) {
    using F = typename Cv::F;
    const uint32_t w = blockIdx.x;
    uint8_t* tx = scratch + (size_t)w * 2 * blockDim.x * Cv::kXyzzBytes;
    uint8_t* tu = tx + (size_t)blockDim.x * Cv::kXyzzBytes;
    Xyzz<F> x, u, q;
    set_identity(x);
    set_identity(u);
    for (uint32_t k = threadIdx.x; k < tw2; k += blockDim.x) {
        const size_t r = (size_t)w * tw2 + k;
        load_xyzz(q, part_x + r * Cv::kXyzzBytes);
        add(x, q);
        load_xyzz(q, part_u + r * Cv::kXyzzBytes);
        add(u, q);
    }
    store_xyzz(tx + (size_t)threadIdx.x * Cv::kXyzzBytes, x);
    store_xyzz(tu + (size_t)threadIdx.x * Cv::kXyzzBytes, u);
    __syncthreads();
    for (uint32_t s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            load_xyzz(x, tx + (size_t)threadIdx.x * Cv::kXyzzBytes);
            load_xyzz(q, tx + (size_t)(threadIdx.x + s) * Cv::kXyzzBytes);
            add(x, q);
            store_xyzz(tx + (size_t)threadIdx.x * Cv::kXyzzBytes, x);
            load_xyzz(u, tu + (size_t)threadIdx.x * Cv::kXyzzBytes);
            load_xyzz(q, tu + (size_t)(threadIdx.x + s) * Cv::kXyzzBytes);
            add(u, q);
            store_xyzz(tu + (size_t)threadIdx.x * Cv::kXyzzBytes, u);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        load_xyzz(x, tx);
        load_xyzz(u, tu);
        for (int i = 0; i < log_chunk; i++) {
            Xyzz<F> d;
            dbl(d, u);
            u = d;
        }
        add(x, u);
        store_xyzz(window_sums + (size_t)w * Cv::kXyzzBytes, x);
    }
}

// dst[g] += src[g] over all buckets (the bucket sums of two batches of points)
template <class Cv>
__global__ void msm_merge_buckets_kernel(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, uint32_t nb) {
    using F = typename Cv::F;
    for (uint32_t g = blockIdx.x * blockDim.x + threadIdx.x; g < nb; g += gridDim.x * blockDim.x) {
        Xyzz<F> a, b;
        load_xyzz(b, src + (size_t)g * Cv::kXyzzBytes);
        if (is_identity(b)) continue;
        load_xyzz(a, dst + (size_t)g * Cv::kXyzzBytes);
        add(a, b);
        store_xyzz(dst + (size_t)g * Cv::kXyzzBytes, a);
    }
}

// ------------------------------------------------------------------ layout conversion
// reference host records (x, y, bool infinity + pad) -> packed (all-zero = infinity)
template <int kCoordWords>
__global__ void pack_ref_points_kernel(const uint64_t* __restrict__ in, size_t n, uint64_t* __restrict__ out) {
    constexpr int kIn = kCoordWords + 1;  // + flag word
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const uint64_t* r = in + i * kIn;
        bool inf = (r[kCoordWords] & 0xff) != 0;
#pragma unroll
        for (int k = 0; k < kCoordWords; k++) out[i * kCoordWords + k] = inf ? 0ull : r[k];
    }
}

// ------------------------------------------------------------------ fixed base
// out_i = k_i * G with a byte comb: table[j][d] = d * 2^(8j) * G (affine).
template <class Cv>
__device__ void affine_from_xyzz_dev(Affine<typename Cv::F>& a, const Xyzz<typename Cv::F>& p);

template <class M>
__device__ void finv_dev(Fe<M>& r, const Fe<M>& a) {
    // a^(m-2), left-to-right square and multiply over the fixed exponent
    Fe<M> acc;
    fset_one(acc);
#pragma unroll
    for (int limb = 7; limb >= 0; limb--) {
        const uint32_t word = limb == 0 ? M::m(0) - 2u : M::m(limb);
        for (int bit = 31; bit >= 0; bit--) {
            fsqr(acc, acc);
            if ((word >> bit) & 1u) fmul(acc, acc, a);
        }
    }
    r = acc;
}
__device__ __forceinline__ void finv_dev(Fp2& r, const Fp2& a) {
    Fp n, t, ni;
    fsqr(n, a.c0);
    fsqr(t, a.c1);
    fadd(n, n, t);
    finv_dev(ni, n);
    fmul(r.c0, a.c0, ni);
    fmul(t, a.c1, ni);
    fneg(r.c1, t);
}

template <class Cv>
__global__ void fixed_base_kernel(const uint8_t* __restrict__ table, const Fr* __restrict__ scalars, size_t n, uint8_t* __restrict__ out) {
    using F = typename Cv::F;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        Fr s;
        fload_nc(s, scalars + i);
        ffrom_mont(s, s);
        Xyzz<F> acc;
        set_identity(acc);
        for (int j = 0; j < 32; j++) {
            uint32_t d = (s.v[0] & 0xffu);
#pragma unroll
            for (int k = 0; k < 7; k++) s.v[k] = __funnelshift_r(s.v[k], s.v[k + 1], 8);
            s.v[7] >>= 8;
            if (d) {
                Affine<F> a;
                load_affine(a, table + ((size_t)j * 256 + d) * Cv::kAffineBytes);
                madd(acc, a);
            }
        }
        uint8_t* o = out + i * Cv::kAffineBytes;
        Affine<F> r;
        if (is_identity(acc)) {
            fset_zero(r.x);
            fset_zero(r.y);
        } else {
            F zi, zzi;
            finv_dev(zi, acc.zz);
            fmul(r.x, acc.x, zi);
            finv_dev(zzi, acc.zzz);
            fmul(r.y, acc.y, zzi);
        }
        fstore(o, r.x);
        fstore(o + sizeof(F), r.y);
    }
}

// out[j n + i] = 2^(c j) P_i (packed affine) for the entries j in [j0, j1) of
// the window tables of a fixed set of bases (all-zero records stay the
// identity): one point per thread, starting from entry j0 - 1 (P_i itself,
// written as entry 0, when j0 = 0), c doublings and one inversion per entry.
// A build is one launch per entry, so that no block holds an SM for long and
// proofs running beside a build get SMs as its blocks retire.
template <class Cv>
__global__ void window_tables_kernel(const uint8_t* __restrict__ pts, size_t n, int c, int j0, int j1, uint8_t* __restrict__ out) {
    using F = typename Cv::F;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    Affine<F> a;
    if (j0 == 0) {
        load_affine(a, pts + i * Cv::kAffineBytes);
        fstore(out + i * Cv::kAffineBytes, a.x);
        fstore(out + i * Cv::kAffineBytes + sizeof(F), a.y);
        j0 = 1;
    } else {
        load_affine(a, out + ((size_t)(j0 - 1) * n + i) * Cv::kAffineBytes);
    }
    const bool inf = fis_zero(a.x) && fis_zero(a.y);
    Xyzz<F> cur, d;
    cur.x = a.x;
    cur.y = a.y;
    fset_one(cur.zz);
    fset_one(cur.zzz);
    for (int j = j0; j < j1; j++) {
        Affine<F> r;
        if (inf) {
            fset_zero(r.x);
            fset_zero(r.y);
        } else {
            for (int t = 0; t < c; t++) {
                dbl(d, cur);
                cur = d;
            }
            // 1 / zz = zzz / (zz zzz), 1 / zzz = zz / (zz zzz): one inversion
            F q, qi, zi, zzi;
            fmul(q, cur.zz, cur.zzz);
            finv_dev(qi, q);
            fmul(zi, cur.zzz, qi);
            fmul(zzi, cur.zz, qi);
            fmul(r.x, cur.x, zi);
            fmul(r.y, cur.y, zzi);
        }
        uint8_t* o = out + ((size_t)j * n + i) * Cv::kAffineBytes;
        fstore(o, r.x);
        fstore(o + sizeof(F), r.y);
    }
}

// ================================================================== host side
template <class Cv>
struct HostCurve;
template <>
struct HostCurve<G1> {
    using F = zkh::Fe;
    static constexpr int kWords = 4;  // u64 words per coordinate
};
template <>
struct HostCurve<G2> {
    using F = zkh::Fp2;
    static constexpr int kWords = 8;
};

template <class HF>
static void host_load(HF& f, const uint64_t* w);
template <>
void host_load<zkh::Fe>(zkh::Fe& f, const uint64_t* w) { std::memcpy(f.v, w, 32); }
template <>
void host_load<zkh::Fp2>(zkh::Fp2& f, const uint64_t* w) { std::memcpy(f.c0.v, w, 32); std::memcpy(f.c1.v, w + 4, 32); }
template <class HF>
static void host_store(uint64_t* w, const HF& f);
template <>
void host_store<zkh::Fe>(uint64_t* w, const zkh::Fe& f) { std::memcpy(w, f.v, 32); }
template <>
void host_store<zkh::Fp2>(uint64_t* w, const zkh::Fp2& f) { std::memcpy(w, f.c0.v, 32); std::memcpy(w + 4, f.c1.v, 32); }

// Horner combine of W window sums (XYZZ records), then affine; out = x || y
template <class Cv>
static void host_combine(const uint64_t* windows, int W, int c, uint64_t* out_affine) {
    using HF = typename HostCurve<Cv>::F;
    constexpr int kw = HostCurve<Cv>::kWords;
    zkh::Xyzz<HF> res, s, d;
    zkh::set_identity(res);
    for (int w = W - 1; w >= 0; w--) {
        for (int i = 0; i < c; i++) {
            zkh::dbl(d, res);
            res = d;
        }
        const uint64_t* r = windows + (size_t)w * 4 * kw;
        host_load(s.x, r);
        host_load(s.y, r + kw);
        host_load(s.zz, r + 2 * kw);
        host_load(s.zzz, r + 3 * kw);
        zkh::add(res, s);
    }
    HF x, y;
    zkh::to_affine(x, y, res);
    host_store(out_affine, x);
    host_store(out_affine + kw, y);
}

static inline unsigned grid_for(size_t work, int threads, int cap) {
    size_t b = (work + threads - 1) / threads;
    if (b < 1) b = 1;
    return (unsigned)std::min<size_t>(b, (size_t)cap);
}

struct LaunchCounter {
    int n = 0;
    void operator++(int) { n++; }
};

// Scratch of the bucket phase (sort + accumulate + fixup), reused by every batch.
struct SortScratch {
    uint32_t *counts, *offsets, *cursors, *tile_sums, *keys, *digits, *first_bucket, *last_bucket, *max_span;
    uint8_t *part_first, *part_last;
};
template <class Cv>
static SortScratch take_sort_scratch(Arena& ar, const MsmPlan& P) {
    SortScratch S;
    S.counts = ar.take<uint32_t>(P.nb + 1);
    S.offsets = ar.take<uint32_t>(P.nb + 1);
    S.cursors = ar.take<uint32_t>(P.nb);
    S.tile_sums = ar.take<uint32_t>(P.tiles);
    S.keys = ar.take<uint32_t>(std::max<size_t>(P.max_keys, 1));
    S.digits = ar.take<uint32_t>(std::max<size_t>(P.max_keys, 1));
    S.part_first = ar.take<uint8_t>(P.max_segs * Cv::kXyzzBytes);
    S.part_last = ar.take<uint8_t>(P.max_segs * Cv::kXyzzBytes);
    S.first_bucket = ar.take<uint32_t>(P.max_segs);
    S.last_bucket = ar.take<uint32_t>(P.max_segs);
    S.max_span = ar.take<uint32_t>(1);
    return S;
}
template <class Cv>
static size_t sort_scratch_bytes(const MsmPlan& P) {
    size_t b = Arena::round((P.nb + 1) * 4) * 2 + Arena::round(P.nb * 4) + Arena::round(P.tiles * 4);
    b += 2 * Arena::round(std::max<size_t>(P.max_keys, 1) * 4);
    b += 2 * Arena::round(P.max_segs * Cv::kXyzzBytes) + 2 * Arena::round(P.max_segs * 4) + Arena::round(4);
    return b;
}

struct ReduceScratch {
    uint8_t *chunk_acc, *chunk_run, *part_x, *part_u, *win_tmp;
    uint8_t *pre_x, *pre_u, *pre_tmp;  // msm_window_pre_kernel (windows with many group results)
};
// blocks per window of msm_window_pre_kernel, 0 when the window kernel alone is short
template <class Cv>
static uint32_t window_pre_blocks(const MsmPlan& P) {
    return P.tw2 > 2 * (uint32_t)win_threads<Cv>() ? (P.tw2 + kWinPre - 1) / kWinPre : 0;
}
template <class Cv>
static ReduceScratch take_reduce_scratch(Arena& ar, const MsmPlan& P) {
    ReduceScratch R;
    R.chunk_acc = ar.take<uint8_t>((size_t)P.W * P.tw * Cv::kXyzzBytes);
    R.chunk_run = ar.take<uint8_t>((size_t)P.W * P.tw * Cv::kXyzzBytes);
    R.part_x = ar.take<uint8_t>((size_t)P.W * P.tw2 * Cv::kXyzzBytes);
    R.part_u = ar.take<uint8_t>((size_t)P.W * P.tw2 * Cv::kXyzzBytes);
    R.win_tmp = ar.take<uint8_t>((size_t)P.W * 2 * win_threads<Cv>() * Cv::kXyzzBytes);
    const size_t pre = (size_t)P.W * window_pre_blocks<Cv>(P);
    R.pre_x = ar.take<uint8_t>(std::max<size_t>(pre, 1) * Cv::kXyzzBytes);
    R.pre_u = ar.take<uint8_t>(std::max<size_t>(pre, 1) * Cv::kXyzzBytes);
    R.pre_tmp = ar.take<uint8_t>(std::max<size_t>(2 * pre * 256, 1) * Cv::kXyzzBytes);
    return R;
}
template <class Cv>
static size_t reduce_scratch_bytes(const MsmPlan& P) {
    size_t b = 2 * Arena::round((size_t)P.W * P.tw * Cv::kXyzzBytes);
    b += 2 * Arena::round((size_t)P.W * P.tw2 * Cv::kXyzzBytes);
    b += Arena::round((size_t)P.W * 2 * win_threads<Cv>() * Cv::kXyzzBytes);
    const size_t pre = (size_t)P.W * window_pre_blocks<Cv>(P);
    b += 2 * Arena::round(std::max<size_t>(pre, 1) * Cv::kXyzzBytes);
    b += Arena::round(std::max<size_t>(2 * pre * 256, 1) * Cv::kXyzzBytes);
    return b;
}

// Signed digits and the counting sort of n scalars into S (keys grouped by
// bucket, offsets).  Records phase events 0..2.
template <class Cv>
static int msm_sort_phase(DeviceContext* ctx, cudaStream_t st, const void* d_scalars, size_t n, const MsmPlan& P,
                          const SortScratch& S, LaunchCounter& lc) {
    cudaEvent_t* ph = ctx->phase;
    const int sms = ctx->num_sms;
    ZK_TRY_CUDA(cudaEventRecord(ph[0], st));
    ZK_TRY_CUDA(cudaMemsetAsync(S.counts, 0, (P.nb + 1) * sizeof(uint32_t), st));
    if (P.agg)
        msm_count_kernel<true><<<grid_for(n, 256, sms * 16), 256, 0, st>>>((const Fr*)d_scalars, n, P.c, P.W, P.wstride, S.counts,
                                                                            S.digits);
    else
        msm_count_kernel<false><<<grid_for(n, 256, sms * 16), 256, 0, st>>>((const Fr*)d_scalars, n, P.c, P.W, P.wstride, S.counts,
                                                                             S.digits);
    lc++;
    ZK_TRY_CUDA(cudaEventRecord(ph[1], st));
    scan_tile_sums_kernel<<<P.tiles, 1024, 0, st>>>(S.counts, P.nb, S.tile_sums);
    lc++;
    scan_tiles_kernel<<<1, 1024, 0, st>>>(S.tile_sums, P.tiles);
    lc++;
    scan_finish_kernel<<<P.tiles, 1024, 0, st>>>(S.counts, P.nb, S.tile_sums, S.offsets, S.cursors);
    lc++;
    ZK_TRY_CUDA(cudaEventRecord(ph[2], st));
    {
        const uint32_t bpw = (uint32_t)((n + 255) / 256);
        if (P.agg)
            msm_scatter_kernel<true><<<bpw * (uint32_t)P.W, 256, 0, st>>>(S.digits, n, P.wstride, P.kstride, bpw, S.cursors, S.keys);
        else
            msm_scatter_kernel<false><<<bpw * (uint32_t)P.W, 256, 0, st>>>(S.digits, n, P.wstride, P.kstride, bpw, S.cursors, S.keys);
    }
    lc++;
    ZK_TRY_CUDA(cudaGetLastError());
    return ZK_OK;
}

// Accumulate + fixup of the sorted keys in S into `buckets` (the sums of the
// nonempty buckets; S.offsets tells which).  d_points must hold the packed
// points when `points_ready` is recorded.  Records phase events 3..5.
template <class Cv>
static int msm_accumulate_phase(DeviceContext* ctx, cudaStream_t st, const void* d_points, const MsmPlan& P, const SortScratch& S,
                                uint8_t* buckets, cudaEvent_t points_ready, LaunchCounter& lc, uint32_t idx_lo = 0,
                                uint32_t idx_hi = 0xffffffffu) {
    cudaEvent_t* ph = ctx->phase;
    ZK_TRY_CUDA(cudaMemsetAsync(S.first_bucket, 0xff, P.max_segs * sizeof(uint32_t), st));
    ZK_TRY_CUDA(cudaMemsetAsync(S.last_bucket, 0xff, P.max_segs * sizeof(uint32_t), st));
    ZK_TRY_CUDA(cudaMemsetAsync(S.max_span, 0, sizeof(uint32_t), st));
    if (points_ready) ZK_TRY_CUDA(cudaStreamWaitEvent(st, points_ready, 0));
    ZK_TRY_CUDA(cudaEventRecord(ph[3], st));
    {
        const int threads = 128;
        unsigned blocks = (unsigned)((P.max_segs + threads - 1) / threads);
        if (blocks < 1) blocks = 1;
        msm_accumulate_kernel<Cv><<<blocks, threads, 0, st>>>(S.keys, S.offsets, P.nb, (const uint8_t*)d_points, P.seg, buckets,
                                                               S.part_first, S.part_last, S.first_bucket, S.last_bucket, idx_lo,
                                                               idx_hi, S.max_span);
        lc++;
    }
    ZK_TRY_CUDA(cudaEventRecord(ph[4], st));
    {
        // grid-stride: a round with no work (past the widest cut bucket) is a short launch
        const unsigned blocks = grid_for(P.max_segs, 128, ctx->num_sms * 16);
        for (uint64_t stride = 1; stride < P.max_segs; stride <<= 1) {
            msm_fixup_round_kernel<Cv><<<blocks, 128, 0, st>>>(S.offsets, S.first_bucket, S.last_bucket, P.max_segs, P.seg, stride,
                                                                S.part_first, S.part_last, S.max_span);
            lc++;
        }
        msm_fixup_final_kernel<Cv><<<(P.nb + 255) / 256, 256, 0, st>>>(S.offsets, P.nb, P.seg, S.part_first, S.part_last, buckets);
        lc++;
    }
    ZK_TRY_CUDA(cudaEventRecord(ph[5], st));
    ZK_TRY_CUDA(cudaGetLastError());
    return ZK_OK;
}

// ------------------------------------------------------------------ batch-affine accumulation (G1)
// Rounds of pairwise affine additions (msm_affine.cuh) when the buckets are
// full enough to pay for them: at least 8 keys per bucket on average and 2^20
// keys.  ZK_MSM_BATCH_AFFINE=0 turns them off, =1 forces them.
static constexpr bool kBaDefault = false;  // on only when ZK_MSM_BATCH_AFFINE=1 until it beats the serial accumulation
static void ba_plan(MsmPlan& P, size_t key_bound, bool g2, int num_sms) {
    P.ba = 0;
    P.key_bound = key_bound;
    if (g2) return;
    const char* env = getenv("ZK_MSM_BATCH_AFFINE");
    const bool want = env && *env ? atoi(env) != 0 : (kBaDefault && key_bound >= ((size_t)1 << 20) && key_bound >= 8 * (size_t)P.nb);
    if (!want || key_bound == 0) return;
    P.ba = kBaRounds;
    P.ba_left = (key_bound >> kBaRounds) + P.nb + 1;
    P.ba_seg = pow2_clamp((double)P.ba_left / ((double)std::max(num_sms, 1) * 512.0), 16, 128);
    P.max_segs = std::max(P.max_segs, (P.ba_left + P.ba_seg - 1) / P.ba_seg);
}

struct BaScratch {
    uint32_t* off[2];         // level offsets (nb + 1), alternating
    uint8_t* pts[2];          // level points: levels 1 and 3 in pts[0]; the dense level 0 and level 2 in pts[1]
    Fp* prefix;               // running products before each regular pair
    Fp* totals;               // per-thread products, turned into their inverses
    Fp* tree;                 // product-tree nodes and upper levels
    unsigned long long* pairs;  // regular pair additions per round, then the elements left (4 words)
};
static size_t ba_bound(const MsmPlan& P, size_t key_bound, int level) { return (key_bound >> level) + P.nb + 1; }
// threads of a pass over `outputs` positions: whole warps of 32 kBaItems positions
static size_t ba_threads(size_t outputs) { return (outputs + 32 * kBaItems - 1) / (32 * kBaItems) * 32; }
static size_t ba_tree_elems(size_t n) {  // nodes of every level plus the upper levels' values
    size_t e = 0;
    while (n > 1) {
        const size_t blocks = (n + kTreeLeaves - 1) / kTreeLeaves;
        e += blocks * 2 * kTreeLeaves + blocks;
        n = blocks;
    }
    return e + 1;
}
static size_t ba_scratch_bytes(const MsmPlan& P, size_t key_bound) {
    if (!P.ba) return 0;
    const size_t b1 = ba_bound(P, key_bound, 1), b0 = std::max(key_bound, ba_bound(P, key_bound, 2)), nt = ba_threads(b1);
    return 2 * Arena::round((size_t)(P.nb + 1) * 4) + Arena::round(b1 * 64) + Arena::round(b0 * 64) + Arena::round(b1 * 32) +
           Arena::round(nt * 32) + Arena::round(ba_tree_elems(nt) * 32) + Arena::round(4 * 8);
}
static BaScratch take_ba_scratch(Arena& ar, const MsmPlan& P, size_t key_bound) {
    BaScratch B{};
    if (!P.ba) return B;
    const size_t b1 = ba_bound(P, key_bound, 1), b0 = std::max(key_bound, ba_bound(P, key_bound, 2)), nt = ba_threads(b1);
    B.off[0] = ar.take<uint32_t>(P.nb + 1);
    B.off[1] = ar.take<uint32_t>(P.nb + 1);
    B.pts[0] = ar.take<uint8_t>(b1 * 64);
    B.pts[1] = ar.take<uint8_t>(b0 * 64);
    B.prefix = ar.take<Fp>(b1);
    B.totals = ar.take<Fp>(nt);
    B.tree = ar.take<Fp>(ba_tree_elems(nt));
    B.pairs = ar.take<unsigned long long>(4);
    return B;
}

// vals[0 .. n) <- their inverses (all nonzero): product tree, one inversion, back down
static int batch_invert(cudaStream_t st, Fp* vals, size_t n, Fp* tree, LaunchCounter& lc) {
    struct Level { Fp* vals; Fp* nodes; size_t n; };
    Level lv[8];
    int L = 0;
    lv[0].vals = vals;
    lv[0].n = n;
    Fp* cur = tree;
    while (lv[L].n > 1) {
        const size_t blocks = (lv[L].n + kTreeLeaves - 1) / kTreeLeaves;
        lv[L].nodes = cur;
        cur += blocks * 2 * kTreeLeaves;
        lv[L + 1].vals = cur;
        lv[L + 1].n = blocks;
        cur += blocks;
        bt_up_kernel<<<(unsigned)blocks, 256, 0, st>>>(lv[L].vals, lv[L].n, lv[L].nodes, lv[L + 1].vals);
        lc++;
        L++;
        if (L >= 7) { set_error("batch inversion: %zu values exceed the tree depth", n); return ZK_ERR_RANGE; }
    }
    bt_invert_kernel<<<1, 32, 0, st>>>(lv[L].vals);
    lc++;
    for (int l = L - 1; l >= 0; l--) {
        bt_down_kernel<<<(unsigned)lv[l + 1].n, 256, 0, st>>>(lv[l].nodes, lv[l + 1].vals, lv[l].n, lv[l].vals);
        lc++;
    }
    ZK_TRY_CUDA(cudaGetLastError());
    return ZK_OK;
}

// Batch-affine rounds over the sorted keys, then the XYZZ accumulation and
// fixup over the level they leave (G1).  Same contract as
// msm_accumulate_phase; phase event 3..4 spans the rounds and the accumulation.
static int ba_accumulate_phase(DeviceContext* ctx, cudaStream_t st, const void* d_points, const MsmPlan& P, const SortScratch& S,
                               const BaScratch& B, size_t key_bound, uint8_t* buckets, cudaEvent_t points_ready, LaunchCounter& lc) {
    cudaEvent_t* ph = ctx->phase;
    ZK_TRY_CUDA(cudaMemsetAsync(S.first_bucket, 0xff, P.max_segs * sizeof(uint32_t), st));
    ZK_TRY_CUDA(cudaMemsetAsync(S.last_bucket, 0xff, P.max_segs * sizeof(uint32_t), st));
    ZK_TRY_CUDA(cudaMemsetAsync(S.max_span, 0, sizeof(uint32_t), st));
    ZK_TRY_CUDA(cudaMemsetAsync(B.pairs, 0, 4 * 8, st));
    if (points_ready) ZK_TRY_CUDA(cudaStreamWaitEvent(st, points_ready, 0));
    ZK_TRY_CUDA(cudaEventRecord(ph[3], st));
    const uint32_t* off_in = S.offsets;
    const uint8_t* pts_in = (const uint8_t*)d_points;
    for (int r = 0; r < P.ba; r++) {
        // level r + 1 goes to pts[0] (odd levels) or pts[1] (even; level 0 too)
        uint32_t* off_out = B.off[r & 1];
        uint8_t* pts_out = B.pts[r & 1];
        // the next level's offsets: exclusive scan of ceil(c_g / 2^(r + 1))
        ba_level_counts_kernel<<<grid_for(P.nb, 256, ctx->num_sms * 8), 256, 0, st>>>(S.offsets, P.nb, r + 1, S.counts);
        scan_tile_sums_kernel<<<P.tiles, 1024, 0, st>>>(S.counts, P.nb, S.tile_sums);
        scan_tiles_kernel<<<1, 1024, 0, st>>>(S.tile_sums, P.tiles);
        scan_finish_kernel<<<P.tiles, 1024, 0, st>>>(S.counts, P.nb, S.tile_sums, off_out, S.cursors);
        for (int k = 0; k < 4; k++) lc++;
        const size_t nt = ba_threads(ba_bound(P, key_bound, r + 1));
        const unsigned blocks = (unsigned)((nt + kBaThreads - 1) / kBaThreads);
        if (r == 0)
            ba_pass_a_kernel<true><<<blocks, kBaThreads, 0, st>>>(S.keys, (const uint8_t*)d_points, B.pts[1], off_in, nullptr, off_out,
                                                                  P.nb, B.prefix, B.totals, nt, B.pairs + r);
        else
            ba_pass_a_kernel<false><<<blocks, kBaThreads, 0, st>>>(nullptr, nullptr, nullptr, off_in, pts_in, off_out, P.nb, B.prefix,
                                                                   B.totals, nt, B.pairs + r);
        lc++;
        ZK_TRY(batch_invert(st, B.totals, nt, B.tree, lc));
        if (r == 0) pts_in = B.pts[1];  // the dense level 0 written by pass A
        ba_pass_b_kernel<<<blocks, kBaThreads, 0, st>>>(off_in, pts_in, off_out, P.nb, B.prefix, B.totals, nt, pts_out);
        lc++;
        off_in = off_out;
        pts_in = pts_out;
    }
    ZK_TRY_CUDA(cudaMemcpyAsync(B.pairs + 3, off_in + P.nb, sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));  // elements left
    {
        const size_t segs = (P.ba_left + P.ba_seg - 1) / P.ba_seg;
        const unsigned blocks = (unsigned)std::max<size_t>(1, (segs + 127) / 128);
        msm_accumulate_kernel<G1, true><<<blocks, 128, 0, st>>>(nullptr, off_in, P.nb, pts_in, P.ba_seg, buckets, S.part_first,
                                                                 S.part_last, S.first_bucket, S.last_bucket, 0, 0xffffffffu,
                                                                 S.max_span);
        lc++;
    }
    ZK_TRY_CUDA(cudaEventRecord(ph[4], st));
    {
        const size_t segs = (P.ba_left + P.ba_seg - 1) / P.ba_seg;
        const unsigned blocks = grid_for(segs, 128, ctx->num_sms * 16);
        for (uint64_t stride = 1; stride < segs; stride <<= 1) {
            msm_fixup_round_kernel<G1><<<blocks, 128, 0, st>>>(off_in, S.first_bucket, S.last_bucket, segs, P.ba_seg, stride,
                                                                S.part_first, S.part_last, S.max_span);
            lc++;
        }
        msm_fixup_final_kernel<G1><<<(P.nb + 255) / 256, 256, 0, st>>>(off_in, P.nb, P.ba_seg, S.part_first, S.part_last, buckets);
        lc++;
    }
    ZK_TRY_CUDA(cudaEventRecord(ph[5], st));
    ZK_TRY_CUDA(cudaGetLastError());
    return ZK_OK;
}

template <class Cv>
static int msm_bucket_phase(DeviceContext* ctx, cudaStream_t st, const void* d_points, const void* d_scalars, size_t n,
                            const MsmPlan& P, const SortScratch& S, uint8_t* buckets, cudaEvent_t points_ready, LaunchCounter& lc) {
    ZK_TRY(msm_sort_phase<Cv>(ctx, st, d_scalars, n, P, S, lc));
    return msm_accumulate_phase<Cv>(ctx, st, d_points, P, S, buckets, points_ready, lc);
}

// Running sums over the buckets of every window; writes W XYZZ window sums.
// offsets == nullptr: every bucket holds its sum (the identity when empty).
// Records phase events 6..7.
template <class Cv>
static int msm_reduce_phase(DeviceContext* ctx, cudaStream_t st, const MsmPlan& P, const uint32_t* offsets, const uint8_t* buckets,
                            const ReduceScratch& R, uint8_t* windows_dev, LaunchCounter& lc) {
    cudaEvent_t* ph = ctx->phase;
    {
        uint32_t total = (uint32_t)P.W * P.tw;
        msm_reduce_kernel<Cv><<<(total + 127) / 128, 128, 0, st>>>(offsets, buckets, P.W, P.B, P.chunk, P.tw, R.chunk_acc, R.chunk_run);
        lc++;
        uint32_t total2 = (uint32_t)P.W * P.tw2;
        msm_reduce2_kernel<Cv><<<(total2 + 127) / 128, 128, 0, st>>>(R.chunk_acc, R.chunk_run, P.W, P.tw, P.chunk2, P.tw2, R.part_x,
                                                                      R.part_u);
        lc++;
    }
    ZK_TRY_CUDA(cudaEventRecord(ph[6], st));
    const uint32_t bpw = window_pre_blocks<Cv>(P);
    if (bpw) {
        msm_window_pre_kernel<Cv><<<dim3((unsigned)P.W * bpw, 2), 256, 0, st>>>(R.part_x, R.part_u, P.tw2, bpw, R.pre_tmp, R.pre_x,
                                                                                R.pre_u);
        lc++;
        msm_window_kernel<Cv><<<P.W, win_threads<Cv>(), 0, st>>>(R.pre_x, R.pre_u, bpw, 31 - __builtin_clz(P.chunk), R.win_tmp,
                                                                 windows_dev);
    } else {
        msm_window_kernel<Cv><<<P.W, win_threads<Cv>(), 0, st>>>(R.part_x, R.part_u, P.tw2, 31 - __builtin_clz(P.chunk), R.win_tmp,
                                                                 windows_dev);
    }
    lc++;
    ZK_TRY_CUDA(cudaEventRecord(ph[7], st));
    ZK_TRY_CUDA(cudaGetLastError());
    return ZK_OK;
}

// Bucket sort + accumulate + reduce; writes W XYZZ window sums to `windows_dev`.
template <class Cv>
static int msm_pipeline(DeviceContext* ctx, cudaStream_t st, const void* d_points, const void* d_scalars, size_t n,
                        const MsmPlan& P, Arena& ar, uint8_t* windows_dev, cudaEvent_t points_ready, LaunchCounter& lc,
                        uint32_t** total_keys_dev, unsigned long long** ba_stats_dev = nullptr) {
    const SortScratch S = take_sort_scratch<Cv>(ar, P);
    *total_keys_dev = S.offsets + P.nb;
    uint8_t* buckets = ar.take<uint8_t>((size_t)P.nb * Cv::kXyzzBytes);
    const ReduceScratch R = take_reduce_scratch<Cv>(ar, P);
    const BaScratch B = take_ba_scratch(ar, P, P.key_bound);
    if (ba_stats_dev) *ba_stats_dev = P.ba ? B.pairs : nullptr;
    ZK_TRY(msm_sort_phase<Cv>(ctx, st, d_scalars, n, P, S, lc));
    if (P.ba && std::is_same<Cv, G1>::value)
        ZK_TRY(ba_accumulate_phase(ctx, st, d_points, P, S, B, P.key_bound, buckets, points_ready, lc));
    else
        ZK_TRY(msm_accumulate_phase<Cv>(ctx, st, d_points, P, S, buckets, points_ready, lc));
    return msm_reduce_phase<Cv>(ctx, st, P, S.offsets, buckets, R, windows_dev, lc);
}

template <class Cv>
static size_t pipeline_bytes(const MsmPlan& P) {
    return sort_scratch_bytes<Cv>(P) + Arena::round((size_t)P.nb * Cv::kXyzzBytes) + reduce_scratch_bytes<Cv>(P) +
           ba_scratch_bytes(P, P.key_bound);
}

// Host inputs from n >= kPipelineMinPoints: kBatches batches of points (a short
// first one, so that accumulation starts early).  The copy stream lands each
// batch's scalars and points in turn; the auxiliary stream sorts a batch as
// soon as its scalars land; the work stream accumulates and fixes it up into
// its own bucket array as soon as its points land, while later batches are
// still crossing PCIe and being sorted.  The arrays are merged (one XYZZ
// addition per bucket and extra batch) before the one reduce.  Unpipelined, the
// accumulate waited for all 1.6 GB of a 2^24 MSM to land.
static constexpr size_t kPipelineMinPoints = (size_t)1 << 20;
static constexpr int kBatches = 3;
static constexpr double kBatchFrac[kBatches] = {0.25, 0.375, 0.375};

template <class Cv>
static int msm_run_host_pipelined(DeviceContext* ctx, cudaStream_t st, const void* h_points, const void* h_scalars, size_t n,
                                  uint64_t* out_affine) {
    MsmStats& stats = msm_stats();
    size_t nk[kBatches], off[kBatches];
    {
        size_t o = 0;
        for (int k = 0; k < kBatches; k++) {
            size_t len = k == kBatches - 1 ? n - o : std::min(n - o, ((size_t)(kBatchFrac[k] * (double)n) + 255) & ~(size_t)255);
            off[k] = o;
            nk[k] = len;
            o += len;
        }
    }
    cudaStream_t cs = ctx->copy_stream, as = ctx->aux_stream;
    cudaEvent_t* ev = ctx->batch_ev;  // batch k: [3k] scalars landed, [3k + 1] points landed, [3k + 2] keys sorted
    ZK_TRY(ensure_pinned(ctx, 4096));
    uint32_t* hist_host = (uint32_t*)ctx->pinned;
    ZK_TRY(scratch_begin(ctx, st));
    ScopedEvent t0, t1;
    ZK_TRY_CUDA(cudaEventCreate(&t0.e));
    ZK_TRY_CUDA(cudaEventCreate(&t1.e));
    ZK_TRY_CUDA(cudaEventRecord(t0.e, st));
    // inputs in the stream-ordered pool (the arena is sized after the plan)
    PoolBuffer pts_buf, sc_buf, hist_buf;
    ZK_TRY_CUDA(pts_buf.alloc(n * Cv::kAffineBytes, st));
    ZK_TRY_CUDA(sc_buf.alloc(n * 32, st));
    ZK_TRY_CUDA(hist_buf.alloc(256 * sizeof(uint32_t), st));
    uint8_t* d_pts = (uint8_t*)pts_buf.p;
    Fr* d_sc = (Fr*)sc_buf.p;
    uint32_t* hist_dev = (uint32_t*)hist_buf.p;
    ZK_TRY_CUDA(cudaEventRecord(ctx->ev_a, st));  // after the previous users of the scratch, and the allocations
    ZK_TRY_CUDA(cudaStreamWaitEvent(cs, ctx->ev_a, 0));
    ZK_TRY_CUDA(cudaStreamWaitEvent(as, ctx->ev_a, 0));
    for (int k = 0; k < kBatches; k++) {  // in arrival order on one copy engine
        ZK_TRY_CUDA(cudaMemcpyAsync(d_sc + off[k], (const uint8_t*)h_scalars + off[k] * 32, nk[k] * 32, cudaMemcpyHostToDevice, cs));
        ZK_TRY_CUDA(cudaEventRecord(ev[3 * k], cs));
        ZK_TRY_CUDA(cudaMemcpyAsync(d_pts + off[k] * Cv::kAffineBytes, (const uint8_t*)h_points + off[k] * Cv::kAffineBytes,
                                    nk[k] * Cv::kAffineBytes, cudaMemcpyHostToDevice, cs));
        ZK_TRY_CUDA(cudaEventRecord(ev[3 * k + 1], cs));
    }
    // the plan from the first batch's scalars
    ZK_TRY_CUDA(cudaStreamWaitEvent(st, ev[0], 0));
    ZK_TRY_CUDA(cudaMemsetAsync(hist_dev, 0, 256 * sizeof(uint32_t), st));
    msm_bitlen_hist_kernel<<<grid_for(nk[0], 256, ctx->num_sms * 4), 256, 0, st>>>(d_sc, nk[0], hist_dev);
    ZK_TRY_CUDA(cudaMemcpyAsync(hist_host, hist_dev, 256 * sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    ZK_TRY_CUDA(cudaStreamSynchronize(st));
    uint32_t hist[256];
    for (int b = 0; b < 256; b++) hist[b] = (uint32_t)std::min<double>(4e9, (double)hist_host[b] * (double)n / (double)nk[0]);
    MsmPlan P = make_plan(n, std::is_same<Cv, G2>::value, hist, ctx->num_sms, false);
    // The batches are sized by the trivial key bound below: a narrow window
    // chosen from small first-batch scalars (many windows) could push that past
    // the 32-bit key space, so such a plan gives way to the full-width one.
    bool fits = true;
    for (int k = 0; k < kBatches; k++) fits = fits && nk[k] * (size_t)P.W <= kMaxKeys;
    if (!fits) P = make_plan(n, std::is_same<Cv, G2>::value, nullptr, ctx->num_sms);
    // per batch, any scalar may have all W digits nonzero: the later batches'
    // histograms are not looked at, so their key bound is the trivial one
    MsmPlan Pb[kBatches];
    int kmax = 0;  // the batch with the most keys: the batch-affine scratch (shared, work stream) is sized for it
    for (int k = 0; k < kBatches; k++) {
        Pb[k] = P;
        Pb[k].max_keys = nk[k] * (size_t)P.W;
        Pb[k].max_segs = std::max<size_t>(1, (Pb[k].max_keys + P.seg - 1) / P.seg);
        ba_plan(Pb[k], Pb[k].max_keys, std::is_same<Cv, G2>::value, ctx->num_sms);
        if (Pb[k].max_keys > Pb[kmax].max_keys) kmax = k;
    }
    stats.window_bits = P.c;
    stats.num_windows = P.W;

    const size_t bucket_bytes = (size_t)P.nb * Cv::kXyzzBytes;
    size_t need = Arena::round((size_t)P.W * Cv::kXyzzBytes) + Arena::round(kBatches * sizeof(uint32_t)) + reduce_scratch_bytes<Cv>(P);
    for (int k = 0; k < kBatches; k++) need += sort_scratch_bytes<Cv>(Pb[k]) + Arena::round(bucket_bytes);
    need += ba_scratch_bytes(Pb[kmax], Pb[kmax].key_bound);
    ZK_TRY(ensure_scratch(ctx, need));  // may synchronise the device (growth only)
    ZK_TRY(ensure_pinned(ctx, (size_t)P.W * Cv::kXyzzBytes + 64));
    Arena ar;
    ar.base = (char*)ctx->scratch;
    uint8_t* windows_dev = ar.take<uint8_t>((size_t)P.W * Cv::kXyzzBytes);
    uint32_t* keys_total = ar.take<uint32_t>(kBatches);
    SortScratch S[kBatches];
    uint8_t* buckets[kBatches];
    for (int k = 0; k < kBatches; k++) {
        S[k] = take_sort_scratch<Cv>(ar, Pb[k]);
        buckets[k] = ar.take<uint8_t>(bucket_bytes);
    }
    const ReduceScratch R = take_reduce_scratch<Cv>(ar, P);
    const BaScratch B = take_ba_scratch(ar, Pb[kmax], Pb[kmax].key_bound);
    LaunchCounter lc;
    for (int k = 0; k < kBatches; k++) {  // sorts, on the auxiliary stream
        ZK_TRY_CUDA(cudaStreamWaitEvent(as, ev[3 * k], 0));
        ZK_TRY(msm_sort_phase<Cv>(ctx, as, d_sc + off[k], nk[k], Pb[k], S[k], lc));
        ZK_TRY_CUDA(cudaEventRecord(ev[3 * k + 2], as));
    }
    // empty buckets must read as the identity (all-zero XYZZ) for the merge;
    // cleared while the work stream still waits for the first batch
    for (int k = 0; k < kBatches; k++) ZK_TRY_CUDA(cudaMemsetAsync(buckets[k], 0, bucket_bytes, st));
    for (int k = 0; k < kBatches; k++) {  // accumulates, on the work stream
        ZK_TRY_CUDA(cudaStreamWaitEvent(st, ev[3 * k + 2], 0));
        if (Pb[k].ba && std::is_same<Cv, G1>::value)
            ZK_TRY(ba_accumulate_phase(ctx, st, d_pts + off[k] * Cv::kAffineBytes, Pb[k], S[k], B, Pb[k].key_bound, buckets[k],
                                       ev[3 * k + 1], lc));
        else
            ZK_TRY(msm_accumulate_phase<Cv>(ctx, st, d_pts + off[k] * Cv::kAffineBytes, Pb[k], S[k], buckets[k], ev[3 * k + 1], lc));
        ZK_TRY_CUDA(cudaMemcpyAsync(keys_total + k, S[k].offsets + P.nb, sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));
    }
    for (int k = 1; k < kBatches; k++) {
        msm_merge_buckets_kernel<Cv><<<grid_for(P.nb, 128, ctx->num_sms * 8), 128, 0, st>>>(buckets[0], buckets[k], P.nb);
        lc++;
    }
    ZK_TRY(msm_reduce_phase<Cv>(ctx, st, P, nullptr, buckets[0], R, windows_dev, lc));
    ZK_TRY_CUDA(cudaMemcpyAsync(ctx->pinned, windows_dev, (size_t)P.W * Cv::kXyzzBytes, cudaMemcpyDeviceToHost, st));
    uint32_t* keys_host = (uint32_t*)((char*)ctx->pinned + (size_t)P.W * Cv::kXyzzBytes);
    ZK_TRY_CUDA(cudaMemcpyAsync(keys_host, keys_total, kBatches * sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    ZK_TRY_CUDA(cudaEventRecord(ctx->phase[8], st));
    ZK_TRY_CUDA(cudaEventRecord(t1.e, st));
    ZK_TRY(scratch_end(ctx, st));
    ZK_TRY_CUDA(cudaStreamSynchronize(st));
    float ms_all = 0;
    cudaEventElapsedTime(&ms_all, t0.e, t1.e);
    // phase times of the last batch (its sort ran on the auxiliary stream) and the reduce
    for (int i = 0; i < 8; i++) cudaEventElapsedTime(&stats.phase_ms[i], ctx->phase[i], ctx->phase[i + 1]);
    stats.kernel_launches = lc.n;
    stats.accumulate_ms = stats.phase_ms[3];
    stats.total_device_ms = ms_all;
    stats.bucket_adds = 0;
    for (int k = 0; k < kBatches; k++) stats.bucket_adds += keys_host[k];
    host_combine<Cv>((const uint64_t*)ctx->pinned, P.W, P.c, out_affine);
    return ZK_OK;
}

// MSM over fixed bases with precomputed window tables (window_tables_kernel):
// the W digits of scalar i select the multiples 2^(c w) P_i, so every window
// shares one set of 2^(c-1) buckets and one reduce, and c can be wider than a
// plain MSM affords (the bucket reduction is paid once, not W times).
template <class Cv>
static int msm_tables_run(int device, cudaStream_t st, const uint8_t* tables, size_t n_total, int c, int W, size_t lo, size_t hi,
                          const void* d_scalars, uint64_t* out_affine) {
    constexpr int kw = HostCurve<Cv>::kWords;
    MsmStats& stats = msm_stats();
    stats = MsmStats();
    if (hi <= lo) {
        std::memset(out_affine, 0, 2 * kw * 8);
        return ZK_OK;
    }
    if (hi > n_total || (size_t)W * n_total >= 0x80000000ull || c < 2 || c > 24 || (size_t)W * c < 255) {
        set_error("msm tables: bad range or shape (n %zu, slice [%zu, %zu), c %d, W %d)", n_total, lo, hi, c, W);
        return ZK_ERR_RANGE;
    }
    const size_t n = hi - lo;
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    std::lock_guard<std::mutex> lock(ctx->mu);
    const double sms = (double)std::max(ctx->num_sms, 1);
    MsmPlan P;
    P.c = c;
    P.W = W;
    P.B = 1u << (c - 1);
    P.nb = P.B;
    P.wstride = 0;
    P.kstride = n_total;
    P.max_keys = n * (size_t)W;
    P.seg = pow2_clamp((double)P.max_keys / (sms * 512.0), 16, 128);
    P.max_segs = std::max<size_t>(1, (P.max_keys + P.seg - 1) / P.seg);
    P.tiles = (P.nb + 1 + kScanTile - 1) / kScanTile;
    P.agg = false;
    MsmPlan Pr = P;  // the reduce sees one window
    Pr.W = 1;
    Pr.chunk = std::min<uint32_t>(P.B, pow2_clamp((double)P.B / (sms * 256.0), 2, 32));
    Pr.tw = P.B / Pr.chunk;
    Pr.chunk2 = std::min<uint32_t>(Pr.tw, pow2_clamp((double)Pr.tw / (sms * 64.0), 2, 16));
    Pr.tw2 = Pr.tw / Pr.chunk2;
    stats.window_bits = c;
    stats.num_windows = W;
    ba_plan(P, P.max_keys, std::is_same<Cv, G2>::value, ctx->num_sms);
    const size_t need = Arena::round(Cv::kXyzzBytes) + sort_scratch_bytes<Cv>(P) + Arena::round((size_t)P.nb * Cv::kXyzzBytes) +
                        reduce_scratch_bytes<Cv>(Pr) + ba_scratch_bytes(P, P.key_bound);
    ZK_TRY(ensure_scratch(ctx, need));
    ZK_TRY(ensure_pinned(ctx, Cv::kXyzzBytes + 64));
    Arena ar;
    ar.base = (char*)ctx->scratch;
    uint8_t* windows_dev = ar.take<uint8_t>(Cv::kXyzzBytes);
    const SortScratch S = take_sort_scratch<Cv>(ar, P);
    uint8_t* buckets = ar.take<uint8_t>((size_t)P.nb * Cv::kXyzzBytes);
    const ReduceScratch R = take_reduce_scratch<Cv>(ar, Pr);
    const BaScratch B = take_ba_scratch(ar, P, P.key_bound);
    LaunchCounter lc;
    ScopedEvent t0, t1;
    ZK_TRY_CUDA(cudaEventCreate(&t0.e));
    ZK_TRY_CUDA(cudaEventCreate(&t1.e));
    ZK_TRY(scratch_begin(ctx, st));
    ZK_TRY_CUDA(cudaEventRecord(t0.e, st));
    ZK_TRY(msm_sort_phase<Cv>(ctx, st, d_scalars, n, P, S, lc));
    if (P.ba && std::is_same<Cv, G1>::value)
        ZK_TRY(ba_accumulate_phase(ctx, st, tables + lo * Cv::kAffineBytes, P, S, B, P.key_bound, buckets, nullptr, lc));
    else
        ZK_TRY(msm_accumulate_phase<Cv>(ctx, st, tables + lo * Cv::kAffineBytes, P, S, buckets, nullptr, lc));
    ZK_TRY(msm_reduce_phase<Cv>(ctx, st, Pr, S.offsets, buckets, R, windows_dev, lc));
    ZK_TRY_CUDA(cudaMemcpyAsync(ctx->pinned, windows_dev, Cv::kXyzzBytes, cudaMemcpyDeviceToHost, st));
    uint32_t* keys_host = (uint32_t*)((char*)ctx->pinned + Cv::kXyzzBytes);
    ZK_TRY_CUDA(cudaMemcpyAsync(keys_host, S.offsets + P.nb, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    ZK_TRY_CUDA(cudaEventRecord(ctx->phase[8], st));
    ZK_TRY_CUDA(cudaEventRecord(t1.e, st));
    ZK_TRY(scratch_end(ctx, st));
    ZK_TRY_CUDA(cudaStreamSynchronize(st));
    float ms_all = 0;
    cudaEventElapsedTime(&ms_all, t0.e, t1.e);
    for (int i = 0; i < 8; i++) cudaEventElapsedTime(&stats.phase_ms[i], ctx->phase[i], ctx->phase[i + 1]);
    stats.kernel_launches = lc.n;
    stats.accumulate_ms = stats.phase_ms[3];
    stats.total_device_ms = ms_all;
    stats.bucket_adds = *keys_host;
    host_combine<Cv>((const uint64_t*)ctx->pinned, 1, c, out_affine);
    return ZK_OK;
}

// Window width for precomputed tables of n bases: minimise the mixed additions
// (n ceil(255 / c), 10 Fp mul each) plus one bucket reduction (2^(c-1) x 30).
// ZK_H_TABLE_BITS (8..22) overrides the choice for tables built afterwards.
void g1_window_tables_shape(size_t n, int* c_out, int* W_out) {
    int best = 12;
    double best_cost = 1e300;
    const char* env = getenv("ZK_H_TABLE_BITS");
    if (env && atoi(env) >= 8 && atoi(env) <= 22) {
        *c_out = atoi(env);
        *W_out = (255 + *c_out - 1) / *c_out;
        return;
    }
    for (int c = 8; c <= 22; c++) {
        const double W = (255 + c - 1) / c;
        const double cost = (double)n * W * 10.0 + (double)(1u << (c - 1)) * 30.0;
        if (cost < best_cost) { best_cost = cost; best = c; }
    }
    *c_out = best;
    *W_out = (255 + best - 1) / best;
}

int g1_window_tables_build(int device, cudaStream_t st, const void* d_points, size_t n, int c, int W, void* d_out) {
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    if (!n) return ZK_OK;
    const unsigned blocks = (unsigned)((n + 127) / 128);
    for (int j = 0; j < W; j++)  // entries 0 and 1 in the first launch
        if (j != 1) {
            window_tables_kernel<G1><<<blocks, 128, 0, st>>>((const uint8_t*)d_points, n, c, j, j == 0 ? std::min(W, 2) : j + 1,
                                                             (uint8_t*)d_out);
            ZK_TRY_CUDA(cudaGetLastError());
        }
    return ZK_OK;
}

int g1_window_tables_msm(int device, cudaStream_t st, const void* tables, size_t n_total, int c, int W, size_t lo, size_t hi,
                         const void* d_scalars, uint64_t* out_affine) {
    return msm_tables_run<G1>(device, st, (const uint8_t*)tables, n_total, c, W, lo, hi, d_scalars, out_affine);
}

// Several MSMs over one vector of device scalars (the witness of a proof, for
// the A, B1, B2 and L queries): one bit-length histogram, one plan and one
// counting sort, then an accumulate + reduce per point set (G1 or G2 packed
// affine).  idx_range (optional, 2 per set): set k uses the scalars
// [lo, hi) only, against its points 0 .. hi - lo.
int msm_shared_scalars_run(DeviceContext* ctx, cudaStream_t st, const void* d_scalars, size_t n, int n_sets, const void* const* d_points,
                           const int* is_g2, const uint32_t* idx_range, uint64_t* const* outs, float* set_ms) {
    MsmStats& stats = msm_stats();
    stats = MsmStats();
    for (int k = 0; k < n_sets; k++) {
        std::memset(outs[k], 0, is_g2[k] ? 128 : 64);
        if (set_ms) set_ms[k] = 0.f;
    }
    if (n == 0 || n_sets == 0) return ZK_OK;
    if (n > kMaxPassPoints || n_sets > 8) {
        set_error("msm: %zu points (at most %zu) or %d point sets (at most 8) out of range", n, kMaxPassPoints, n_sets);
        return ZK_ERR_RANGE;
    }
    ZK_TRY(check_forced_window(n, false));
    ZK_TRY_CUDA(cudaSetDevice(ctx->device));
    std::lock_guard<std::mutex> lock(ctx->mu);
    const double sms = (double)std::max(ctx->num_sms, 1);
    ZK_TRY(ensure_pinned(ctx, 4096));
    uint32_t* hist_host = (uint32_t*)ctx->pinned;
    ZK_TRY(scratch_begin(ctx, st));
    {
        PoolBuffer hist_buf;
        ZK_TRY_CUDA(hist_buf.alloc(256 * sizeof(uint32_t), st));
        uint32_t* hist_dev = (uint32_t*)hist_buf.p;
        ZK_TRY_CUDA(cudaMemsetAsync(hist_dev, 0, 256 * sizeof(uint32_t), st));
        msm_bitlen_hist_kernel<<<grid_for(n, 256, ctx->num_sms * 4), 256, 0, st>>>((const Fr*)d_scalars, n, hist_dev);
        ZK_TRY_CUDA(cudaMemcpyAsync(hist_host, hist_dev, 256 * sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    }
    ZK_TRY_CUDA(cudaStreamSynchronize(st));
    uint32_t hist[256];
    std::memcpy(hist, hist_host, sizeof hist);
    const MsmPlan P = make_plan(n, false, hist, ctx->num_sms);  // the sort, and the G1 accumulates
    ZK_TRY(check_key_bound(P, hist));
    MsmPlan P2 = P;                                           // G2 accumulates: shorter segments
    P2.seg = pow2_clamp((double)plan_key_bound(P, hist) / (sms * 512.0), 8, 64);
    P2.max_segs = std::max<size_t>(1, (plan_key_bound(P, hist) + P2.seg - 1) / P2.seg);
    stats.window_bits = P.c;
    stats.num_windows = P.W;

    // The sets share the keys but nothing else: each gets its own partial
    // slots, buckets and reduce scratch and runs on its own stream, so their
    // chains of dependent additions (fixup rounds, running sums, window sums
    // over a witness's few full buckets) overlap instead of queueing.
    auto set_bytes = [&](bool g2) {
        const MsmPlan& Q = g2 ? P2 : P;
        const size_t xb = g2 ? G2::kXyzzBytes : G1::kXyzzBytes;
        return 2 * Arena::round(Q.max_segs * xb) + 2 * Arena::round(Q.max_segs * 4) + Arena::round(4) +
               Arena::round((size_t)P.nb * xb) + (g2 ? reduce_scratch_bytes<G2>(P2) : reduce_scratch_bytes<G1>(P));
    };
    size_t need = sort_scratch_bytes<G1>(P) + Arena::round((size_t)n_sets * P.W * G2::kXyzzBytes);
    for (int k = 0; k < n_sets; k++) need += set_bytes(is_g2[k] != 0);
    ZK_TRY(ensure_scratch(ctx, need));
    ZK_TRY(ensure_pinned(ctx, (size_t)n_sets * P.W * G2::kXyzzBytes + 64));
    ZK_TRY(ensure_set_streams(ctx));
    Arena ar;
    ar.base = (char*)ctx->scratch;
    const SortScratch S = take_sort_scratch<G1>(ar, P);
    uint8_t* windows = ar.take<uint8_t>((size_t)n_sets * P.W * G2::kXyzzBytes);
    SortScratch Sk[8];
    uint8_t* buckets[8];
    ReduceScratch Rk[8];
    for (int k = 0; k < n_sets; k++) {
        const bool g2 = is_g2[k] != 0;
        const MsmPlan& Q = g2 ? P2 : P;
        const size_t xb = g2 ? G2::kXyzzBytes : G1::kXyzzBytes;
        Sk[k] = S;  // the keys and offsets are shared
        Sk[k].part_first = ar.take<uint8_t>(Q.max_segs * xb);
        Sk[k].part_last = ar.take<uint8_t>(Q.max_segs * xb);
        Sk[k].first_bucket = ar.take<uint32_t>(Q.max_segs);
        Sk[k].last_bucket = ar.take<uint32_t>(Q.max_segs);
        Sk[k].max_span = ar.take<uint32_t>(1);
        buckets[k] = ar.take<uint8_t>((size_t)P.nb * xb);
        Rk[k] = g2 ? take_reduce_scratch<G2>(ar, P2) : take_reduce_scratch<G1>(ar, P);
    }
    LaunchCounter lc;
    ScopedEvent ev[9], done[8];
    for (int k = 0; k <= n_sets; k++) ZK_TRY_CUDA(cudaEventCreate(&ev[k].e));
    for (int k = 0; k < n_sets; k++) ZK_TRY_CUDA(cudaEventCreateWithFlags(&done[k].e, cudaEventDisableTiming));
    ZK_TRY(msm_sort_phase<G1>(ctx, st, d_scalars, n, P, S, lc));
    ZK_TRY_CUDA(cudaEventRecord(ev[0].e, st));
    for (int k = 0; k < n_sets; k++) {
        cudaStream_t ss = ctx->set_stream[k];
        ZK_TRY_CUDA(cudaStreamWaitEvent(ss, ev[0].e, 0));
        uint8_t* win = windows + (size_t)k * P.W * G2::kXyzzBytes;
        const uint32_t ilo = idx_range ? idx_range[2 * k] : 0u, ihi = idx_range ? idx_range[2 * k + 1] : 0xffffffffu;
        if (is_g2[k]) {
            ZK_TRY(msm_accumulate_phase<G2>(ctx, ss, d_points[k], P2, Sk[k], buckets[k], nullptr, lc, ilo, ihi));
            ZK_TRY(msm_reduce_phase<G2>(ctx, ss, P2, S.offsets, buckets[k], Rk[k], win, lc));
        } else {
            ZK_TRY(msm_accumulate_phase<G1>(ctx, ss, d_points[k], P, Sk[k], buckets[k], nullptr, lc, ilo, ihi));
            ZK_TRY(msm_reduce_phase<G1>(ctx, ss, P, S.offsets, buckets[k], Rk[k], win, lc));
        }
        ZK_TRY_CUDA(cudaEventRecord(ev[k + 1].e, ss));
        ZK_TRY_CUDA(cudaEventRecord(done[k].e, ss));
    }
    for (int k = 0; k < n_sets; k++) ZK_TRY_CUDA(cudaStreamWaitEvent(st, done[k].e, 0));
    ZK_TRY_CUDA(cudaMemcpyAsync(ctx->pinned, windows, (size_t)n_sets * P.W * G2::kXyzzBytes, cudaMemcpyDeviceToHost, st));
    uint32_t* keys_host = (uint32_t*)((char*)ctx->pinned + (size_t)n_sets * P.W * G2::kXyzzBytes);
    ZK_TRY_CUDA(cudaMemcpyAsync(keys_host, S.offsets + P.nb, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    ZK_TRY(scratch_end(ctx, st));
    ZK_TRY_CUDA(cudaStreamSynchronize(st));
    if (set_ms)  // each set from the end of the shared sort (the sets overlap)
        for (int k = 0; k < n_sets; k++) cudaEventElapsedTime(&set_ms[k], ev[0].e, ev[k + 1].e);
    stats.kernel_launches = lc.n;
    stats.bucket_adds = (long long)*keys_host * n_sets;
    for (int k = 0; k < n_sets; k++) {
        const uint64_t* win = (const uint64_t*)((const uint8_t*)ctx->pinned + (size_t)k * P.W * G2::kXyzzBytes);
        if (is_g2[k]) host_combine<G2>(win, P.W, P.c, outs[k]);
        else host_combine<G1>(win, P.W, P.c, outs[k]);
    }
    return ZK_OK;
}

template <class Cv>
static void host_add_affine(const uint64_t* a, const uint64_t* b, uint64_t* out);

// Full MSM.  src_points / src_scalars are device pointers (host_inputs == 0)
// or host pointers (host_inputs == 1, copied in chunks on the copy stream).
// ref_layout: points are reference records (72 / 136 B) rather than packed.
// More than kMaxPassPoints points run as consecutive passes whose affine
// results are added on the host, so that no pass outgrows the 32-bit key space.
template <class Cv>
static int msm_run(int device, cudaStream_t user_stream, const void* src_points, const void* src_scalars, size_t n,
                   bool host_inputs, bool ref_layout, uint64_t* out_affine) {
    constexpr int kw = HostCurve<Cv>::kWords;
    MsmStats& stats = msm_stats();
    stats = MsmStats();
    if (n == 0) {
        std::memset(out_affine, 0, 2 * kw * 8);
        return ZK_OK;
    }
    if (n > kMaxPassPoints) {
        const size_t rec = ref_layout ? Cv::kAffineBytes + 8 : Cv::kAffineBytes;
        uint64_t acc[2 * kw] = {}, part[2 * kw];
        MsmStats sum;
        for (size_t off = 0; off < n; off += kMaxPassPoints) {
            const size_t cnt = std::min(kMaxPassPoints, n - off);
            ZK_TRY(msm_run<Cv>(device, user_stream, (const uint8_t*)src_points + off * rec, (const uint8_t*)src_scalars + off * 32,
                               cnt, host_inputs, ref_layout, part));
            host_add_affine<Cv>(acc, part, acc);
            const MsmStats& s = msm_stats();
            sum.kernel_launches += s.kernel_launches;
            sum.accumulate_ms += s.accumulate_ms;
            sum.total_device_ms += s.total_device_ms;
            sum.bucket_adds += s.bucket_adds;
            sum.ba_pairs += s.ba_pairs;
            sum.ba_left += s.ba_left;
            sum.window_bits = s.window_bits;
            sum.num_windows = s.num_windows;
            for (int i = 0; i < 8; i++) sum.phase_ms[i] += s.phase_ms[i];
        }
        stats = sum;
        std::memcpy(out_affine, acc, sizeof acc);
        return ZK_OK;
    }
    ZK_TRY(check_forced_window(n, std::is_same<Cv, G2>::value));
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    std::lock_guard<std::mutex> lock(ctx->mu);
    cudaStream_t st = user_stream;  // NULL: the legacy default stream
    if (host_inputs && !ref_layout && n >= kPipelineMinPoints)
        return msm_run_host_pipelined<Cv>(ctx, st, src_points, src_scalars, n, out_affine);
    // Window choice from the scalars' bit lengths (a small device pre-pass; the
    // host path copies the scalars first for it).
    ZK_TRY(ensure_pinned(ctx, 4096));
    uint32_t* hist_host = (uint32_t*)ctx->pinned;
    const void* sc_for_hist = src_scalars;
    ZK_TRY(scratch_begin(ctx, st));
    PoolBuffer hist_buf, sc_buf;  // returned to the pool on every exit path, after the queued work
    ZK_TRY_CUDA(hist_buf.alloc(256 * sizeof(uint32_t), st));
    uint32_t* hist_dev = (uint32_t*)hist_buf.p;
    void* sc_copy = nullptr;
    if (host_inputs) {
        ZK_TRY_CUDA(sc_buf.alloc(n * 32, st));
        sc_copy = sc_buf.p;
        ZK_TRY_CUDA(cudaMemcpyAsync(sc_copy, src_scalars, n * 32, cudaMemcpyHostToDevice, st));
        sc_for_hist = sc_copy;
    }
    ZK_TRY_CUDA(cudaMemsetAsync(hist_dev, 0, 256 * sizeof(uint32_t), st));
    msm_bitlen_hist_kernel<<<grid_for(n, 256, ctx->num_sms * 4), 256, 0, st>>>((const Fr*)sc_for_hist, n, hist_dev);
    ZK_TRY_CUDA(cudaMemcpyAsync(hist_host, hist_dev, 256 * sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    ZK_TRY_CUDA(cudaStreamSynchronize(st));
    uint32_t hist[256];
    std::memcpy(hist, hist_host, sizeof hist);
    MsmPlan P = make_plan(n, std::is_same<Cv, G2>::value, hist, ctx->num_sms);
    ZK_TRY(check_key_bound(P, hist));
    ba_plan(P, plan_key_bound(P, hist), std::is_same<Cv, G2>::value, ctx->num_sms);
    stats.window_bits = P.c;
    stats.num_windows = P.W;

    const size_t pt_bytes = n * Cv::kAffineBytes;
    const size_t ref_bytes = ref_layout ? n * (Cv::kAffineBytes + 8) : 0;
    size_t need = pipeline_bytes<Cv>(P) + Arena::round((size_t)P.W * Cv::kXyzzBytes);
    const bool own_points = host_inputs || ref_layout;
    if (own_points) need += Arena::round(pt_bytes);
    if (ref_layout) need += Arena::round(ref_bytes);
    ZK_TRY(ensure_scratch(ctx, need));
    ZK_TRY(ensure_pinned(ctx, (size_t)P.W * Cv::kXyzzBytes + 128));
    Arena ar;
    ar.base = (char*)ctx->scratch;
    uint8_t* windows_dev = ar.take<uint8_t>((size_t)P.W * Cv::kXyzzBytes);
    const void* d_points = src_points;
    const void* d_scalars = src_scalars;
    uint8_t* packed = own_points ? ar.take<uint8_t>(pt_bytes) : nullptr;
    uint8_t* raw = ref_layout ? ar.take<uint8_t>(ref_bytes) : nullptr;
    LaunchCounter lc;

    ScopedEvent t0, t1;
    ZK_TRY_CUDA(cudaEventCreate(&t0.e));
    ZK_TRY_CUDA(cudaEventCreate(&t1.e));
    ZK_TRY_CUDA(cudaEventRecord(t0.e, st));

    cudaEvent_t points_ready = nullptr;
    if (host_inputs) {
        // scalars first on the work stream (the sort needs them); points on the
        // copy stream, overlapped with the decomposition and sort.
        d_scalars = sc_copy;  // copied for the histogram above
        ZK_TRY_CUDA(cudaEventRecord(ctx->ev_a, st));
        ZK_TRY_CUDA(cudaStreamWaitEvent(ctx->copy_stream, ctx->ev_a, 0));
        if (ref_layout) {
            ZK_TRY_CUDA(cudaMemcpyAsync(raw, src_points, ref_bytes, cudaMemcpyHostToDevice, ctx->copy_stream));
            pack_ref_points_kernel<Cv::kAffineBytes / 8><<<grid_for(n, 256, ctx->num_sms * 8), 256, 0, ctx->copy_stream>>>(
                (const uint64_t*)raw, n, (uint64_t*)packed);
            lc++;
        } else {
            ZK_TRY_CUDA(cudaMemcpyAsync(packed, src_points, pt_bytes, cudaMemcpyHostToDevice, ctx->copy_stream));
        }
        ZK_TRY_CUDA(cudaEventRecord(ctx->ev_b, ctx->copy_stream));
        points_ready = ctx->ev_b;
        d_points = packed;
    } else if (ref_layout) {
        pack_ref_points_kernel<Cv::kAffineBytes / 8><<<grid_for(n, 256, ctx->num_sms * 8), 256, 0, st>>>(
            (const uint64_t*)src_points, n, (uint64_t*)packed);
        lc++;
        d_points = packed;
    }

    uint32_t* total_keys_dev = nullptr;
    unsigned long long* ba_dev = nullptr;
    ZK_TRY(msm_pipeline<Cv>(ctx, st, d_points, d_scalars, n, P, ar, windows_dev, points_ready, lc, &total_keys_dev, &ba_dev));
    ZK_TRY_CUDA(cudaMemcpyAsync(ctx->pinned, windows_dev, (size_t)P.W * Cv::kXyzzBytes, cudaMemcpyDeviceToHost, st));
    uint32_t* keys_host = (uint32_t*)((char*)ctx->pinned + (size_t)P.W * Cv::kXyzzBytes);
    ZK_TRY_CUDA(cudaMemcpyAsync(keys_host, total_keys_dev, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    unsigned long long* ba_host = (unsigned long long*)((char*)ctx->pinned + (size_t)P.W * Cv::kXyzzBytes + 64);
    if (ba_dev) ZK_TRY_CUDA(cudaMemcpyAsync(ba_host, ba_dev, 4 * 8, cudaMemcpyDeviceToHost, st));
    ZK_TRY_CUDA(cudaEventRecord(ctx->phase[8], st));
    ZK_TRY_CUDA(cudaEventRecord(t1.e, st));
    ZK_TRY(scratch_end(ctx, st));
    ZK_TRY_CUDA(cudaStreamSynchronize(st));
    float ms_all = 0;
    cudaEventElapsedTime(&ms_all, t0.e, t1.e);
    for (int i = 0; i < 8; i++) cudaEventElapsedTime(&stats.phase_ms[i], ctx->phase[i], ctx->phase[i + 1]);
    stats.kernel_launches = lc.n;
    stats.accumulate_ms = stats.phase_ms[3];
    stats.total_device_ms = ms_all;
    stats.bucket_adds = *keys_host;
    if (ba_dev) {
        stats.ba_pairs = (long long)(ba_host[0] + ba_host[1] + ba_host[2]);
        stats.ba_left = (long long)(ba_host[3] & 0xffffffffull);
    }
    host_combine<Cv>((const uint64_t*)ctx->pinned, P.W, P.c, out_affine);
    return ZK_OK;
}

// ------------------------------------------------------------------ fixed-base tables
template <class Cv>
static int fixed_base_table(DeviceContext* ctx, void** table_dev);

template <class Cv>
static void host_generator(typename HostCurve<Cv>::F& x, typename HostCurve<Cv>::F& y);
template <>
void host_generator<G1>(zkh::Fe& x, zkh::Fe& y) {
    uint64_t one[4] = {1, 0, 0, 0}, two[4] = {2, 0, 0, 0};
    zkh::from_std(zkh::kP, x, one);
    zkh::from_std(zkh::kP, y, two);
}
template <>
void host_generator<G2>(zkh::Fp2& x, zkh::Fp2& y) {
    // EIP-197 G2 generator, standard form (quoted in src/curve/g2.cuh:8-13)
    static const uint64_t X0[4] = {0x46DEBD5CD992F6EDULL, 0x674322D4F75EDADDULL, 0x426A00665E5C4479ULL, 0x1800DEEF121F1E76ULL};
    static const uint64_t X1[4] = {0x97E485B7AEF312C2ULL, 0xF1AA493335A9E712ULL, 0x7260BFB731FB5D25ULL, 0x198E9393920D483AULL};
    static const uint64_t Y0[4] = {0x4CE6CC0166FA7DAAULL, 0xE3D1E7690C43D37BULL, 0x4AAB71808DCB408FULL, 0x12C85EA5DB8C6DEBULL};
    static const uint64_t Y1[4] = {0x55ACDADCD122975BULL, 0xBC4B313370B38EF3ULL, 0xEC9E99AD690C3395ULL, 0x090689D0585FF075ULL};
    zkh::from_std(zkh::kP, x.c0, X0);
    zkh::from_std(zkh::kP, x.c1, X1);
    zkh::from_std(zkh::kP, y.c0, Y0);
    zkh::from_std(zkh::kP, y.c1, Y1);
}

static std::mutex g_table_mu;
static void* g_tables[64][2];

template <class Cv>
static int fixed_base_table(DeviceContext* ctx, void** table_dev) {
    const int which = std::is_same<Cv, G2>::value ? 1 : 0;
    std::lock_guard<std::mutex> lock(g_table_mu);
    if (ctx->device < 0 || ctx->device >= 64) return ZK_ERR_INVALID;
    if (g_tables[ctx->device][which]) {
        *table_dev = g_tables[ctx->device][which];
        return ZK_OK;
    }
    using HF = typename HostCurve<Cv>::F;
    constexpr int kw = HostCurve<Cv>::kWords;
    std::vector<uint64_t> tab((size_t)32 * 256 * 2 * kw, 0);
    HF gx, gy;
    host_generator<Cv>(gx, gy);
    zkh::Xyzz<HF> base, acc, d;
    zkh::from_affine(base, gx, gy);
    for (int j = 0; j < 32; j++) {
        zkh::set_identity(acc);
        for (int k = 1; k < 256; k++) {
            zkh::add(acc, base);
            HF x, y;
            zkh::to_affine(x, y, acc);
            uint64_t* r = &tab[((size_t)j * 256 + k) * 2 * kw];
            host_store(r, x);
            host_store(r + kw, y);
        }
        for (int i = 0; i < 8; i++) {
            zkh::dbl(d, base);
            base = d;
        }
    }
    void* p = nullptr;
    ZK_TRY_CUDA(cudaMalloc(&p, tab.size() * 8));
    ZK_TRY_CUDA(cudaMemcpy(p, tab.data(), tab.size() * 8, cudaMemcpyHostToDevice));
    g_tables[ctx->device][which] = p;
    *table_dev = p;
    return ZK_OK;
}

template <class Cv>
static int fixed_base_run(int device, cudaStream_t user_stream, void* d_out, const void* d_scalars, size_t n) {
    if (n == 0) return ZK_OK;
    if (!d_out || !d_scalars) { set_error("fixed_base: null pointer"); return ZK_ERR_INVALID; }
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    void* table;
    ZK_TRY(fixed_base_table<Cv>(ctx, &table));
    cudaStream_t st = user_stream;  // NULL: the legacy default stream
    fixed_base_kernel<Cv><<<grid_for(n, 128, ctx->num_sms * 8), 128, 0, st>>>((const uint8_t*)table, (const Fr*)d_scalars, n,
                                                                              (uint8_t*)d_out);
    ZK_TRY_CUDA(cudaGetLastError());
    return ZK_OK;
}

// ------------------------------------------------------------------ host point adds
template <class Cv>
static void host_add_affine(const uint64_t* a, const uint64_t* b, uint64_t* out) {
    using HF = typename HostCurve<Cv>::F;
    constexpr int kw = HostCurve<Cv>::kWords;
    auto is_zero_rec = [](const uint64_t* r) {
        for (int i = 0; i < 2 * kw; i++) if (r[i]) return false;
        return true;
    };
    zkh::Xyzz<HF> pa, pb;
    zkh::set_identity(pa);
    zkh::set_identity(pb);
    HF x, y;
    if (!is_zero_rec(a)) { host_load(x, a); host_load(y, a + kw); zkh::from_affine(pa, x, y); }
    if (!is_zero_rec(b)) { host_load(x, b); host_load(y, b + kw); zkh::from_affine(pb, x, y); }
    zkh::add(pa, pb);
    zkh::to_affine(x, y, pa);
    host_store(out, x);
    host_store(out + kw, y);
}

}  // namespace zk

// ================================================================== C ABI (MSM part)
using namespace zk;

extern "C" int zk_msm_g1_device(int device, void* stream, const void* d_points, const void* d_scalars, size_t n, void* out_affine) {
    clear_error();
    if ((n && (!d_points || !d_scalars)) || !out_affine) { set_error("zk_msm_g1_device: null pointer"); return ZK_ERR_INVALID; }
    return msm_run<G1>(device, (cudaStream_t)stream, d_points, d_scalars, n, false, false, (uint64_t*)out_affine);
}
extern "C" int zk_msm_g1_host(int device, void* stream, const void* h_points, const void* h_scalars, size_t n, void* out_affine) {
    clear_error();
    if ((n && (!h_points || !h_scalars)) || !out_affine) { set_error("zk_msm_g1_host: null pointer"); return ZK_ERR_INVALID; }
    return msm_run<G1>(device, (cudaStream_t)stream, h_points, h_scalars, n, true, false, (uint64_t*)out_affine);
}
extern "C" int zk_msm_g2_device(int device, void* stream, const void* d_points, const void* d_scalars, size_t n, void* out_affine) {
    clear_error();
    if ((n && (!d_points || !d_scalars)) || !out_affine) { set_error("zk_msm_g2_device: null pointer"); return ZK_ERR_INVALID; }
    return msm_run<G2>(device, (cudaStream_t)stream, d_points, d_scalars, n, false, false, (uint64_t*)out_affine);
}
extern "C" int zk_msm_g2_host(int device, void* stream, const void* h_points, const void* h_scalars, size_t n, void* out_affine) {
    clear_error();
    if ((n && (!h_points || !h_scalars)) || !out_affine) { set_error("zk_msm_g2_host: null pointer"); return ZK_ERR_INVALID; }
    return msm_run<G2>(device, (cudaStream_t)stream, h_points, h_scalars, n, true, false, (uint64_t*)out_affine);
}

// Reference-shaped: host ref records, result as a ref Jacobian (x, y, one)
template <class Cv>
static int ref_msm(const void* h_points, const void* h_scalars, int n, void* out_jacobian) {
    clear_error();
    constexpr int kw = HostCurve<Cv>::kWords;
    if (n < 0 || !out_jacobian || (n > 0 && (!h_points || !h_scalars))) {
        set_error("msm: invalid arguments (n = %d)", n);
        return ZK_ERR_INVALID;
    }
    uint64_t aff[16];
    ZK_TRY(msm_run<Cv>(-1, nullptr, h_points, h_scalars, (size_t)n, true, true, aff));
    uint64_t* o = (uint64_t*)out_jacobian;
    bool inf = true;
    for (int i = 0; i < 2 * kw; i++) if (aff[i]) inf = false;
    std::memset(o, 0, 3 * kw * 8);
    if (inf) {
        std::memcpy(o + kw, zkh::kP.one, 32);  // identity (0, one, 0)
    } else {
        std::memcpy(o, aff, 2 * kw * 8);
        std::memcpy(o + 2 * kw, zkh::kP.one, 32);  // Z = one (c1 = 0 for G2)
    }
    return ZK_OK;
}

extern "C" int zk_msm_g1(const void* h_points, const void* h_scalars, int n, void* out_jacobian) {
    return ref_msm<G1>(h_points, h_scalars, n, out_jacobian);
}
extern "C" int zk_msm_g2(const void* h_points, const void* h_scalars, int n, void* out_jacobian) {
    return ref_msm<G2>(h_points, h_scalars, n, out_jacobian);
}

extern "C" int zk_g1_fixed_base_device(int device, void* stream, void* d_out, const void* d_scalars, size_t n) {
    clear_error();
    return fixed_base_run<G1>(device, (cudaStream_t)stream, d_out, d_scalars, n);
}
extern "C" int zk_g2_fixed_base_device(int device, void* stream, void* d_out, const void* d_scalars, size_t n) {
    clear_error();
    return fixed_base_run<G2>(device, (cudaStream_t)stream, d_out, d_scalars, n);
}

extern "C" int zk_g1_add_affine(const void* a, const void* b, void* out) {
    clear_error();
    if (!a || !b || !out) { set_error("zk_g1_add_affine: null pointer"); return ZK_ERR_INVALID; }
    uint64_t r[8];
    host_add_affine<G1>((const uint64_t*)a, (const uint64_t*)b, r);
    std::memcpy(out, r, 64);
    return ZK_OK;
}
extern "C" int zk_g2_add_affine(const void* a, const void* b, void* out) {
    clear_error();
    if (!a || !b || !out) { set_error("zk_g2_add_affine: null pointer"); return ZK_ERR_INVALID; }
    uint64_t r[16];
    host_add_affine<G2>((const uint64_t*)a, (const uint64_t*)b, r);
    std::memcpy(out, r, 128);
    return ZK_OK;
}

extern "C" int zk_msm_last_stats(zk_msm_stats* out) {
    if (!out) return ZK_ERR_INVALID;
    const MsmStats& s = msm_stats();
    out->kernel_launches = s.kernel_launches;
    out->accumulate_ms = s.accumulate_ms;
    out->total_device_ms = s.total_device_ms;
    out->window_bits = s.window_bits;
    out->num_windows = s.num_windows;
    out->bucket_adds = s.bucket_adds;
    out->batch_affine_pairs = s.ba_pairs;
    out->batch_affine_left = s.ba_left;
    for (int i = 0; i < 8; i++) out->phase_ms[i] = s.phase_ms[i];
    return ZK_OK;
}
