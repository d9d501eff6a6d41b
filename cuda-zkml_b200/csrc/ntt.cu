// ntt.cu -- BN254 Fr NTT / INTT / coset NTT on sm_100a.
//
// Replaces the reference's ntt_gpu (src/ntt/ntt.cu:354-465), which runs a
// bit-reversal scatter, 10 shared-memory stages with per-butterfly
// square-and-multiply twiddles, then one global radix-2 launch per remaining
// stage, each preceded by a host twiddle build and a host-to-device copy.
//
// Here the transform is the in-place four-step (Bailey) decomposition
// n = R_0 R_1 ... R_{P-1}, R_p = 2^r_p <= 256:
//   pass p views each level block of size N_p = R_p R_{p+1} ... as R_p x M_p
//   (M_p = N_p / R_p) and, for every column j2, computes the R_p-point DFT
//   over the rows in shared memory (radix-2 DIF stages, roots of order R_p
//   from a small table), multiplies output k1 by w_{N_p}^(j2 k1), and stores
//   it back to row k1 of the same column.
// After the last pass, element X[f] sits at the mixed-radix digit reversal of
// f; one permutation kernel moves it to natural order and applies any final
// scale (n^-1) and coset factor (g^-f), so the whole transform is P + 1
// launches with 2 (P + 1) streaming passes over HBM.  Inter-pass twiddles
// w_n^e and coset factors come from one table of all n factors up to
// 2^kFullTableMaxLog (one 32-byte read per element in each pass that applies
// them, in place of a Montgomery product), else from two 2^(L/2)-entry tables
// (w^lo * w^(hi 2^h)) held in L2.
//
// A CTA owns C adjacent columns (C = 8: 256-byte contiguous runs per row) or,
// in the last pass (M = 1), C adjacent contiguous sub-transforms, so every
// global access is a full 32-byte sector of a coalesced run.
// The NTT butterfly loop is small enough for the instruction cache with the
// Montgomery multiplication inlined, which measured 9% faster than the
// out-of-line body the MSM kernels use (2^24 forward: 6.07 vs 6.65 ms).
#ifndef ZK_NTT_FMUL_OUTLINE
#define ZK_FMUL_OUTLINE 0
#endif
#include "field.cuh"
#include "host_field.hpp"
#include "runtime.cuh"

#include <atomic>
#include <cstring>
#include <map>
#include <mutex>
#include <memory>
#include <vector>

namespace zk {

static constexpr int kMaxLogR = 8;
static constexpr int kNttThreads = 256;
static constexpr int kTileElems = 2048;  // R * C per CTA (64 KiB of shared memory)

// ------------------------------------------------------------------ tables
// Twiddle and coset factors are read through table_factor: factor(i) =
// lo[i & (2^h - 1)] * hi[i >> h] from two 2^(L/2)-entry tables, or, when h < 0,
// lo[i] from one table of all n factors.  The full tables (built once per size
// up to 2^kFullTableMaxLog, by the same products) trade one Montgomery product
// per factor for a 32-byte load: the transform is IMAD-bound with DRAM ~5% busy.
static constexpr int kFullTableMaxLog = 24;

struct NttDirTables {
    Fr* roots = nullptr;   // w_{2^r}^t for r = 1..8, t < 2^(r-1), concatenated at offset 2^(r-1) - 1
    Fr* tw_lo = nullptr;   // w_n^i, i < 2^h (all i < n when h < 0)
    Fr* tw_hi = nullptr;   // w_n^(i 2^h), i < 2^(L-h)
    int h = 0;
};
struct CosetTables {       // factor(i) = lo[i & (2^h - 1)] * hi[i >> h], or lo[i] when h < 0
    Fr* lo = nullptr;
    Fr* hi = nullptr;
    int h = 0;
};
static int expand_full_table(DeviceContext* ctx, Fr** lo, Fr** hi, int* h, int L);
struct NttTables {
    std::map<int, NttDirTables> dir;            // key: L * 2 + inverse
    std::map<std::vector<uint64_t>, CosetTables> coset;  // key: L, kind, g limbs
};

void release_ntt_tables(DeviceContext* ctx) {
    if (!ctx->ntt) return;
    for (auto& kv : ctx->ntt->dir) {
        cudaFree(kv.second.roots);
        cudaFree(kv.second.tw_lo);
        cudaFree(kv.second.tw_hi);
    }
    for (auto& kv : ctx->ntt->coset) {
        cudaFree(kv.second.lo);
        cudaFree(kv.second.hi);
    }
    delete ctx->ntt;
    ctx->ntt = nullptr;
}

static void host_fr_pow_u64(zkh::Fe& r, const zkh::Fe& a, uint64_t e) {
    uint64_t ee[4] = {e, 0, 0, 0};
    zkh::pow(zkh::kR, r, a, ee);
}

// primitive 2^L-th root of unity: 5^((r-1)/2^L); w_{2^28} = 5^((r-1)/2^28)
// (src/ntt/ntt.cu:43-62), then squared 28 - L times (ntt.cu:64-106)
static zkh::Fe host_root(int L, bool inverse) {
    uint64_t e[4];
    std::memcpy(e, zkh::kR.m, 32);
    e[0] -= 1;
    for (int s = 0; s < 28; s++)
        for (int i = 0; i < 4; i++) e[i] = (e[i] >> 1) | (i < 3 ? e[i + 1] << 63 : 0);
    uint64_t five[4] = {5, 0, 0, 0};
    zkh::Fe g, w;
    zkh::from_std(zkh::kR, g, five);
    zkh::pow(zkh::kR, w, g, e);
    if (inverse) {
        zkh::Fe wi;
        zkh::inv(zkh::kR, wi, w);
        w = wi;
    }
    for (int i = 0; i < 28 - L; i++) zkh::mul(zkh::kR, w, w, w);
    return w;
}

static int upload(Fr** dst, const std::vector<zkh::Fe>& v) {
    ZK_TRY_CUDA(cudaMalloc((void**)dst, v.size() * 32));
    ZK_TRY_CUDA(cudaMemcpy(*dst, v.data(), v.size() * 32, cudaMemcpyHostToDevice));
    return ZK_OK;
}

static void powers(std::vector<zkh::Fe>& out, const zkh::Fe& start, const zkh::Fe& step, size_t count) {
    out.resize(count);
    zkh::Fe cur = start;
    for (size_t i = 0; i < count; i++) {
        out[i] = cur;
        zkh::mul(zkh::kR, cur, cur, step);
    }
}

static int get_dir_tables(DeviceContext* ctx, int L, bool inverse, const NttDirTables** out) {
    if (!ctx->ntt) ctx->ntt = new NttTables();
    int key = L * 2 + (inverse ? 1 : 0);
    auto it = ctx->ntt->dir.find(key);
    if (it != ctx->ntt->dir.end()) {
        *out = &it->second;
        return ZK_OK;
    }
    NttDirTables t;
    t.h = (L + 1) / 2;
    zkh::Fe one = zkh::one(zkh::kR);
    zkh::Fe w = host_root(L, inverse);
    std::vector<zkh::Fe> v;
    powers(v, one, w, (size_t)1 << t.h);
    ZK_TRY(upload(&t.tw_lo, v));
    zkh::Fe wh = w;
    for (int i = 0; i < t.h; i++) zkh::mul(zkh::kR, wh, wh, wh);
    powers(v, one, wh, (size_t)1 << (L - t.h));
    ZK_TRY(upload(&t.tw_hi, v));
    std::vector<zkh::Fe> roots;
    for (int r = 1; r <= kMaxLogR; r++) {
        std::vector<zkh::Fe> p;
        powers(p, one, host_root(r, inverse), (size_t)1 << (r - 1));
        roots.insert(roots.end(), p.begin(), p.end());
    }
    ZK_TRY(upload(&t.roots, roots));
    if (L <= kFullTableMaxLog) ZK_TRY(expand_full_table(ctx, &t.tw_lo, &t.tw_hi, &t.h, L));
    auto res = ctx->ntt->dir.emplace(key, t);
    *out = &res.first->second;
    return ZK_OK;
}

// kind 0: g^i          (forward coset pre-multiplication)
// kind 1: n^-1 g^-i    (inverse coset post-multiplication)
// kind 2: n^-1 g^i     (INTT followed by the coset shift, fused)
// kind 3: g^-i         (inverse coset factor without the n^-1)
static int get_coset_tables(DeviceContext* ctx, int L, int kind, const zkh::Fe& g, const CosetTables** out) {
    if (!ctx->ntt) ctx->ntt = new NttTables();
    std::vector<uint64_t> key = {(uint64_t)L, (uint64_t)kind, g.v[0], g.v[1], g.v[2], g.v[3]};
    auto it = ctx->ntt->coset.find(key);
    if (it != ctx->ntt->coset.end()) {
        *out = &it->second;
        return ZK_OK;
    }
    CosetTables t;
    t.h = (L + 1) / 2;
    zkh::Fe one = zkh::one(zkh::kR), step = g, start = one;
    if (kind == 1 || kind == 3) zkh::inv(zkh::kR, step, g);
    if (kind == 1 || kind == 2) {
        zkh::Fe two, ninv;
        uint64_t s2[4] = {2, 0, 0, 0};
        zkh::from_std(zkh::kR, two, s2);
        zkh::inv(zkh::kR, ninv, two);
        start = one;
        for (int i = 0; i < L; i++) zkh::mul(zkh::kR, start, start, ninv);
    }
    std::vector<zkh::Fe> v;
    powers(v, start, step, (size_t)1 << t.h);
    ZK_TRY(upload(&t.lo, v));
    zkh::Fe sh = step;
    for (int i = 0; i < t.h; i++) zkh::mul(zkh::kR, sh, sh, sh);
    powers(v, one, sh, (size_t)1 << (L - t.h));
    ZK_TRY(upload(&t.hi, v));
    if (L <= kFullTableMaxLog) ZK_TRY(expand_full_table(ctx, &t.lo, &t.hi, &t.h, L));
    auto res = ctx->ntt->coset.emplace(key, t);
    *out = &res.first->second;
    return ZK_OK;
}

// ------------------------------------------------------------------ kernels
__device__ __forceinline__ void table_factor(Fr& f, const Fr* lo, const Fr* hi, int h, uint64_t i) {
    if (h < 0) {  // one table of all n factors
        fload_nc(f, lo + i);
        return;
    }
    Fr a, b;
    fload_nc(a, lo + (i & ((1ull << h) - 1)));
    fload_nc(b, hi + (i >> h));
    fmul(f, a, b);
}

// full[i] = lo[i & (2^h - 1)] * hi[i >> h], i < n: the same product table_factor forms
__global__ void expand_table_kernel(Fr* __restrict__ full, const Fr* __restrict__ lo, const Fr* __restrict__ hi, int h, uint64_t n) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        Fr x;
        table_factor(x, lo, hi, h, i);
        fstore(full + i, x);
    }
}

// Replace the two split tables by the full table of 2^L factors (once per size).
static int expand_full_table(DeviceContext* ctx, Fr** lo, Fr** hi, int* h, int L) {
    const uint64_t n = 1ull << L;
    Fr* full = nullptr;
    ZK_TRY_CUDA(cudaMalloc(&full, n * sizeof(Fr)));
    const unsigned grid = (unsigned)std::min<uint64_t>((n + 255) / 256, (uint64_t)ctx->num_sms * 16);
    expand_table_kernel<<<grid, 256, 0, ctx->stream>>>(full, *lo, *hi, *h, n);
    ZK_TRY_CUDA(cudaGetLastError());
    ZK_TRY_CUDA(cudaStreamSynchronize(ctx->stream));
    cudaFree(*lo);
    cudaFree(*hi);
    *lo = full;
    *hi = nullptr;
    *h = -1;
    return ZK_OK;
}

// K consecutive radix-2 DIF stages (half sizes hh, hh/2, ..., hh/2^(K-1)) on
// groups of 2^K elements held in registers: element t of a group sits at row
// j0 + t s (s = hh / 2^(K-1)), and stage i pairs t with t + 2^(K-1-i).  The
// twiddle of a pair is w_{2h}^qh with h the stage's half size and qh the upper
// element's position mod h, as in one radix-2 stage at a time; K stages cost
// one shared-memory round trip and one barrier instead of K.
template <int K>
__device__ __forceinline__ void dif_stages(Fr* sm, const Fr* sroot, int R, int C, int hh) {
    constexpr int G = 1 << K;
    const int s = hh >> (K - 1);
    for (int g = threadIdx.x; g < (R / G) * C; g += blockDim.x) {
        const int c = g % C, q = g / C;
        const int m = q % s, j0 = (q / s) * 2 * hh + m;
        Fr x[G];
#pragma unroll
        for (int t = 0; t < G; t++) fload(x[t], sm + (j0 + t * s) * C + c);
#pragma unroll
        for (int i = 0; i < K; i++) {
            const int half = 1 << (K - 1 - i);
            const int hi = hh >> i;
#pragma unroll
            for (int t = 0; t < G; t++) {
                if (t & half) continue;
                Fr a = x[t], b = x[t + half];
                fadd(x[t], a, b);
                fsub(x[t + half], a, b);
                const int tix = (m + (t & (half - 1)) * s) * (R / (2 * hi));
                if (tix) {
                    Fr w;
                    fload(w, sroot + tix);
                    fmul(x[t + half], x[t + half], w);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < G; t++) fstore(sm + (j0 + t * s) * C + c, x[t]);
    }
}

// Radix-2 stages held in registers per shared-memory round trip (1..3) and the
// CTAs per SM the passes are compiled for.  Measured at 2^24 (forward): groups of
// 4 at 3 CTAs per SM (76 registers, no spills) 4.92 ms; groups of 8 at 2 CTAs
// (124 registers) 5.07 ms, at 3 CTAs (80 registers, spills) 5.03 ms; groups of
// 8 left unbounded (144 registers, 1 CTA) 7.10 ms; one stage at a time 5.58 ms.
#ifndef ZK_NTT_MAXK
#define ZK_NTT_MAXK 2
#endif
#ifndef ZK_NTT_MINB
#define ZK_NTT_MINB 3
#endif

template <int LOGR>
__global__ void __launch_bounds__(kNttThreads, ZK_NTT_MINB) ntt_pass_kernel(const Fr* __restrict__ src, Fr* __restrict__ dst, int L, int Lp, int C,
                                                               const Fr* __restrict__ roots, const Fr* __restrict__ tw_lo,
                                                               const Fr* __restrict__ tw_hi, int h, const Fr* __restrict__ cs_lo,
                                                               const Fr* __restrict__ cs_hi, int cs_h) {
    constexpr int R = 1 << LOGR;
    extern __shared__ uint4 smem_raw[];
    Fr* sm = reinterpret_cast<Fr*>(smem_raw);
    Fr* sroot = sm + R * C;
    const uint64_t M = 1ull << (Lp - LOGR);
    const uint64_t Np = 1ull << Lp;
    const uint64_t l0 = (uint64_t)blockIdx.x * C;
    const int E = R * C;
    const bool col_major = M >= (uint64_t)C;  // C adjacent columns of one level block

    for (int t = threadIdx.x; t < R / 2; t += blockDim.x) {
        Fr x;
        fload_nc(x, roots + (R / 2 - 1) + t);
        fstore(sroot + t, x);
    }
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int c, j1;
        if (col_major) { c = e % C; j1 = e / C; } else { j1 = e % R; c = e / R; }
        const uint64_t line = l0 + c;
        const uint64_t gi = (line / M) * Np + (line % M) + (uint64_t)j1 * M;
        Fr x;
        fload_nc(x, src + gi);
        if (cs_lo) {  // first pass of a forward coset transform: gi is the natural index
            Fr f;
            table_factor(f, cs_lo, cs_hi, cs_h, gi);
            fmul(x, x, f);
        }
        fstore(sm + j1 * C + c, x);
    }
    __syncthreads();
    // radix-2 DIF stages hh = R/2, R/4, ..., 1, up to ZK_NTT_MAXK at a time in registers
    int hh = R / 2;
    if (ZK_NTT_MAXK >= 3 && LOGR >= 3) {
#pragma unroll 1
        for (; hh >= 4; hh >>= 3) {
            dif_stages<3>(sm, sroot, R, C, hh);
            __syncthreads();
        }
    }
    if (ZK_NTT_MAXK >= 2) {
#pragma unroll 1
        for (; hh >= 2; hh >>= 2) {
            dif_stages<2>(sm, sroot, R, C, hh);
            __syncthreads();
        }
    }
#pragma unroll 1
    for (; hh >= 1; hh >>= 1) {
        dif_stages<1>(sm, sroot, R, C, hh);
        __syncthreads();
    }
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int c, k1;
        if (col_major) { c = e % C; k1 = e / C; } else { k1 = e % R; c = e / R; }
        const uint64_t line = l0 + c;
        const uint64_t j2 = line % M;
        const int kr = LOGR ? (int)(__brev((unsigned)k1) >> (32 - LOGR)) : 0;
        Fr y;
        fload(y, sm + kr * C + c);
        const uint64_t en = (j2 * (uint64_t)k1) << (L - Lp);
        if (en) {
            Fr w;
            table_factor(w, tw_lo, tw_hi, h, en);
            fmul(y, y, w);
        }
        fstore(dst + (line / M) * Np + j2 + (uint64_t)k1 * M, y);
    }
}

// out[f] = src[pos(f)] * factor(f); pos = mixed-radix digit reversal of f.
// mode 0: no factor; 1: constant; 2: table factor.  When `pa`/`pb` are given
// the epilogue is the compute_h pointwise step out = (pa*pb - y) * scale.
struct PermPlan {
    int P;
    int r[4];
};
__global__ void ntt_permute_kernel(const Fr* __restrict__ src, Fr* __restrict__ dst, int L, PermPlan pp, int mode, Fr scale,
                                   const Fr* __restrict__ f_lo, const Fr* __restrict__ f_hi, int fh, const Fr* __restrict__ pa,
                                   const Fr* __restrict__ pb) {
    const uint64_t n = 1ull << L;
    for (uint64_t f = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; f < n; f += (uint64_t)gridDim.x * blockDim.x) {
        uint64_t rem = f, pos = 0;
        int suffix = L;
        for (int p = 0; p < pp.P; p++) {
            const uint64_t k = rem & ((1ull << pp.r[p]) - 1);
            rem >>= pp.r[p];
            suffix -= pp.r[p];
            pos += k << suffix;
        }
        Fr y;
        fload_nc(y, src + pos);
        if (pa) {
            Fr a, b;
            fload_nc(a, pa + f);
            fload_nc(b, pb + f);
            fmul(a, a, b);
            fsub(y, a, y);
        }
        if (mode == 1) {
            fmul(y, y, scale);
        } else if (mode == 2) {
            Fr t;
            table_factor(t, f_lo, f_hi, fh, f);
            fmul(y, y, t);
        }
        fstore(dst + f, y);
    }
}

// ------------------------------------------------------------------ host driver
static PermPlan make_pass_plan(int L) {
    PermPlan pp;
    pp.P = (L + kMaxLogR - 1) / kMaxLogR;
    if (pp.P < 1) pp.P = 1;
    int rem = L;
    for (int p = 0; p < pp.P; p++) {
        int left = pp.P - p;
        pp.r[p] = (rem + left - 1) / left;  // balanced, larger passes first
        rem -= pp.r[p];
    }
    return pp;
}

typedef void (*PassFn)(const Fr*, Fr*, int, int, int, const Fr*, const Fr*, const Fr*, int, const Fr*, const Fr*, int);

static PassFn pass_fn(int logr) {
    switch (logr) {
        case 1: return ntt_pass_kernel<1>;
        case 2: return ntt_pass_kernel<2>;
        case 3: return ntt_pass_kernel<3>;
        case 4: return ntt_pass_kernel<4>;
        case 5: return ntt_pass_kernel<5>;
        case 6: return ntt_pass_kernel<6>;
        case 7: return ntt_pass_kernel<7>;
        case 8: return ntt_pass_kernel<8>;
        default: return nullptr;
    }
}

struct FinalOp {
    int mode = 0;          // 0 none, 1 constant, 2 table
    Fr scale{};
    const CosetTables* tab = nullptr;
    const Fr* pa = nullptr;  // pointwise epilogue operands
    const Fr* pb = nullptr;
};

// Forward/inverse passes from `src` into `buf`, then the permute into `dst`.
// `pre`: optional coset tables applied on the first pass's loads.
static int ntt_core(DeviceContext* ctx, cudaStream_t st, Fr* dst, const Fr* src, Fr* buf, int L, bool inverse, const CosetTables* pre,
                    const FinalOp& fin, int* launches) {
    const uint64_t n = 1ull << L;
    if (L == 0) {  // a one-point transform is the identity (times the final factor)
        PermPlan none;
        none.P = 0;
        ntt_permute_kernel<<<1, 32, 0, st>>>(src, dst, 0, none, fin.mode, fin.scale, fin.tab ? fin.tab->lo : nullptr,
                                             fin.tab ? fin.tab->hi : nullptr, fin.tab ? fin.tab->h : 0, fin.pa, fin.pb);
        (*launches)++;
        ZK_TRY_CUDA(cudaGetLastError());
        return ZK_OK;
    }
    const NttDirTables* T;
    ZK_TRY(get_dir_tables(ctx, L, inverse, &T));
    PermPlan pp = make_pass_plan(L);
    int Lp = L;
    const Fr* in = src;
    for (int p = 0; p < pp.P; p++) {
        const int r = pp.r[p];
        const uint64_t M = 1ull << (Lp - r);
        const uint64_t lines = n >> r;
        int C;  // columns per CTA: R C = kTileElems where the level block allows, at least 8 adjacent
        if (M >= 8) C = (int)std::min<uint64_t>(M, (uint64_t)std::max(8, kTileElems >> r));
        else C = (int)std::min<uint64_t>(lines, (uint64_t)std::max(1, kTileElems >> r));
        const size_t smem = ((size_t)(1 << r) * C + (1 << r) / 2 + 1) * sizeof(Fr);
        PassFn fn = pass_fn(r);
        static bool attr_set[kMaxLogR + 1][64];
        if (!attr_set[r][ctx->device]) {
            ZK_TRY_CUDA(cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
            attr_set[r][ctx->device] = true;
        }
        const unsigned grid = (unsigned)(lines / C);
        fn<<<grid, kNttThreads, smem, st>>>(in, buf, L, Lp, C, T->roots, T->tw_lo, T->tw_hi, T->h, (p == 0 && pre) ? pre->lo : nullptr,
                                            (p == 0 && pre) ? pre->hi : nullptr, pre ? pre->h : 0);
        (*launches)++;
        in = buf;
        Lp -= r;
    }
    const unsigned pgrid = (unsigned)std::min<uint64_t>((n + 255) / 256, (uint64_t)ctx->num_sms * 16);
    ntt_permute_kernel<<<pgrid, 256, 0, st>>>(buf, dst, L, pp, fin.mode, fin.scale, fin.tab ? fin.tab->lo : nullptr,
                                              fin.tab ? fin.tab->hi : nullptr, fin.tab ? fin.tab->h : 0, fin.pa, fin.pb);
    (*launches)++;
    ZK_TRY_CUDA(cudaGetLastError());
    return ZK_OK;
}

static Fr n_inverse_dev(int L) {
    zkh::Fe two, half, s = zkh::one(zkh::kR);
    uint64_t s2[4] = {2, 0, 0, 0};
    zkh::from_std(zkh::kR, two, s2);
    zkh::inv(zkh::kR, half, two);
    for (int i = 0; i < L; i++) zkh::mul(zkh::kR, s, s, half);
    Fr f;
    std::memcpy(f.v, s.v, 32);
    return f;
}

static thread_local int g_ntt_launches = 0;

int ntt_run(int device, cudaStream_t user_stream, void* d_out, const void* d_in, int L, bool inverse, const void* coset_g) {
    if (!d_out || !d_in) { set_error("ntt: null pointer"); return ZK_ERR_INVALID; }
    if (L < 0 || L > ZK_NTT_MAX_LOG) { set_error("ntt: log_n = %d outside [0, %d]", L, ZK_NTT_MAX_LOG); return ZK_ERR_RANGE; }
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    std::lock_guard<std::mutex> lock(ctx->mu);
    cudaStream_t st = user_stream;  // NULL: the legacy default stream
    const uint64_t n = 1ull << L;
    ZK_TRY(ensure_scratch(ctx, n * 32));
    Fr* buf = (Fr*)ctx->scratch;
    const CosetTables* pre = nullptr;
    FinalOp fin;
    zkh::Fe g;
    if (coset_g) std::memcpy(g.v, coset_g, 32);
    if (!inverse) {
        if (coset_g) ZK_TRY(get_coset_tables(ctx, L, 0, g, &pre));
    } else if (coset_g) {
        fin.mode = 2;
        ZK_TRY(get_coset_tables(ctx, L, 1, g, &fin.tab));
    } else {
        fin.mode = 1;
        fin.scale = n_inverse_dev(L);
    }
    g_ntt_launches = 0;
    ZK_TRY(scratch_begin(ctx, st));
    ZK_TRY(ntt_core(ctx, st, (Fr*)d_out, (const Fr*)d_in, buf, L, inverse, pre, fin, &g_ntt_launches));
    return scratch_end(ctx, st);
}

// coset generator g = 5, or 7 when 5^n == 1 (groth16.cu:329-342), and
// (g^n - 1)^-1, the inverse of the vanishing polynomial on the coset
static int coset_shift(int L, zkh::Fe& g, zkh::Fe& zinv) {
    zkh::Fe z, one = zkh::one(zkh::kR);
    uint64_t s5[4] = {5, 0, 0, 0}, s7[4] = {7, 0, 0, 0};
    zkh::from_std(zkh::kR, g, s5);
    auto vanish = [&](const zkh::Fe& gg) {
        zkh::Fe t = gg;
        for (int i = 0; i < L; i++) zkh::mul(zkh::kR, t, t, t);
        zkh::sub(zkh::kR, t, t, one);
        return t;
    };
    z = vanish(g);
    if (zkh::is_zero(z)) {
        zkh::from_std(zkh::kR, g, s7);
        z = vanish(g);
    }
    if (zkh::is_zero(z)) { set_error("compute_h: no valid coset shift"); return ZK_ERR_INVALID; }
    zkh::inv(zkh::kR, zinv, z);
    return ZK_OK;
}

// out = (a b - c) * zinv, elementwise (out may alias any input)
__global__ void h_pointwise_kernel(Fr* out, const Fr* a, const Fr* b, const Fr* c, uint64_t n, Fr zinv) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        Fr x, y, z;
        fload_nc(x, a + i);
        fload_nc(y, b + i);
        fload_nc(z, c + i);
        fmul(x, x, y);
        fsub(x, x, z);
        fmul(x, x, zinv);
        fstore(out + i, x);
    }
}

// ------------------------------------------------------------------ transforms split over parts
// A 2^L-point transform split over N = 2^s parts (one per GPU), m = n / N,
// q = m / N, with two layouts of a part p's m elements:
//   cyclic   local t          <-> global p + N t
//   blocks   local k q + v    <-> global k m + p q + v      (k < N, v < q)
// cyclic -> blocks:  X[k1 m + k2] = sum_j1 w_N^(j1 k1) w^(j1 k2) sum_j2 x[j1 + N j2] w_m^(j2 k2):
//   each part runs the m-point transform of its cyclic elements, an all-to-all
//   sends the k2 in [p' q, p' q + q) to part p', and ntt_cross_kernel mode 0
//   applies w^(j1 k2) to what part j1 sent and the N-point transform over j1.
// blocks -> cyclic:  X[k1 + N k2] = sum_j2 w_m^(j2 k2) w^(j2 k1) sum_j1 w_N^(j1 k1) x[j1 m + j2]:
//   ntt_cross_kernel mode 1 runs the N-point transforms over the local blocks
//   and applies w^(j2 k1); an all-to-all sends block k1 to part k1, which runs
//   the m-point transform of what it gathered (j2 in order).
// One all-to-all per transform; the layouts chain (an INTT from cyclic to
// blocks feeds a coset NTT from blocks back to cyclic).  An optional factor
// f(global index) is applied to the outputs (mode 0) or inputs (mode 1), and
// `scale` (N^-1 for an inverse transform) to the outputs.
struct RootsN {
    Fr w[4];  // w_N^t, t < N / 2
};

template <int LOGN>
__global__ void __launch_bounds__(256) ntt_cross_kernel(const Fr* __restrict__ in, Fr* __restrict__ out, uint64_t q, uint64_t m,
                                                        uint64_t part, int mode, const Fr* __restrict__ tw_lo,
                                                        const Fr* __restrict__ tw_hi, int tw_h, const Fr* __restrict__ f_lo,
                                                        const Fr* __restrict__ f_hi, int f_h, RootsN roots, Fr scale, int has_scale) {
    constexpr int N = 1 << LOGN;
    for (uint64_t v = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; v < q; v += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t j = part * q + v;  // k2 (mode 0) or j2 (mode 1)
        Fr x[N];
#pragma unroll
        for (int a = 0; a < N; a++) fload_nc(x[a], in + a * q + v);
#pragma unroll
        for (int a = 0; a < N; a++) {
            Fr t;
            if (mode == 0) {
                if (a) {  // w^(j1 k2), j1 k2 < N m = n
                    table_factor(t, tw_lo, tw_hi, tw_h, (uint64_t)a * j);
                    fmul(x[a], x[a], t);
                }
            } else if (f_lo) {
                table_factor(t, f_lo, f_hi, f_h, (uint64_t)a * m + j);
                fmul(x[a], x[a], t);
            }
        }
        // N-point DIF over the parts: half sizes N/2 .. 1, outputs in bit-reversed order
#pragma unroll
        for (int h = N / 2; h >= 1; h >>= 1) {
#pragma unroll
            for (int i = 0; i < N; i++) {
                if (i & h) continue;
                Fr s, d;
                fadd(s, x[i], x[i + h]);
                fsub(d, x[i], x[i + h]);
                const int t = (i & (h - 1)) * (N / (2 * h));
                if (t) fmul(d, d, roots.w[t]);
                x[i] = s;
                x[i + h] = d;
            }
        }
#pragma unroll
        for (int pos = 0; pos < N; pos++) {
            const int k = LOGN ? (int)(__brev((unsigned)pos) >> (32 - LOGN)) : 0;
            Fr y = x[pos], t;
            if (mode == 0) {
                if (f_lo) {
                    table_factor(t, f_lo, f_hi, f_h, (uint64_t)k * m + j);
                    fmul(y, y, t);
                }
            } else if (k) {  // w^(j2 k1), j2 k1 < m N = n
                table_factor(t, tw_lo, tw_hi, tw_h, j * (uint64_t)k);
                fmul(y, y, t);
            }
            if (has_scale) fmul(y, y, scale);
            fstore(out + (uint64_t)k * q + v, y);
        }
    }
}

int ntt_cross_run(int device, cudaStream_t st, void* d_out, const void* d_in, int L, int log_parts, int part, bool inverse, int mode,
                  const void* factor_g, bool factor_inverse) {
    if (!d_out || !d_in) { set_error("ntt_cross: null pointer"); return ZK_ERR_INVALID; }
    if (log_parts < 0 || log_parts > 3 || 2 * log_parts > L || L > ZK_NTT_MAX_LOG || part < 0 || part >= (1 << log_parts) ||
        mode < 0 || mode > 1) {
        set_error("ntt_cross: log_n %d, log_parts %d, part %d, mode %d out of range", L, log_parts, part, mode);
        return ZK_ERR_RANGE;
    }
    if (d_out == d_in) { set_error("ntt_cross: d_out must not alias d_in"); return ZK_ERR_INVALID; }
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    std::lock_guard<std::mutex> lock(ctx->mu);
    const NttDirTables* T;
    ZK_TRY(get_dir_tables(ctx, L, inverse, &T));
    const CosetTables* F = nullptr;
    if (factor_g) {
        zkh::Fe g;
        std::memcpy(g.v, factor_g, 32);
        ZK_TRY(get_coset_tables(ctx, L, factor_inverse ? 3 : 0, g, &F));
    }
    const int N = 1 << log_parts;
    const uint64_t m = 1ull << (L - log_parts), q = m >> log_parts;
    RootsN roots;
    const zkh::Fe w = host_root(L, inverse);
    for (int t = 0; t < 4; t++) {
        zkh::Fe r;
        host_fr_pow_u64(r, w, (uint64_t)t * m);  // w_N = w^m
        std::memcpy(roots.w[t].v, r.v, 32);
    }
    Fr scale{};
    int has_scale = 0;
    if (inverse && N > 1) {
        scale = n_inverse_dev(log_parts);
        has_scale = 1;
    }
    const unsigned grid = (unsigned)std::max<uint64_t>(1, std::min<uint64_t>((q + 255) / 256, (uint64_t)ctx->num_sms * 8));
    const Fr* fl = F ? F->lo : nullptr;
    const Fr* fh = F ? F->hi : nullptr;
    const int fhh = F ? F->h : 0;
    switch (log_parts) {
#define ZK_CROSS(S)                                                                                                                    \
    case S:                                                                                                                            \
        ntt_cross_kernel<S><<<grid, 256, 0, st>>>((const Fr*)d_in, (Fr*)d_out, q, m, (uint64_t)part, mode, T->tw_lo, T->tw_hi, T->h, \
                                                  fl, fh, fhh, roots, scale, has_scale);                                              \
        break;
        ZK_CROSS(0)
        ZK_CROSS(1)
        ZK_CROSS(2)
        ZK_CROSS(3)
#undef ZK_CROSS
    }
    ZK_TRY_CUDA(cudaGetLastError());
    return ZK_OK;
}

// compute_h after the matvec (src/prover/groth16.cu:322-383)
int compute_h_run(int device, cudaStream_t user_stream, void* d_h, const void* d_a, const void* d_b, const void* d_c, int L) {
    if (!d_h || !d_a || !d_b || !d_c) { set_error("compute_h: null pointer"); return ZK_ERR_INVALID; }
    if (L < 0 || L > ZK_NTT_MAX_LOG - 1) { set_error("compute_h: log_n = %d out of range", L); return ZK_ERR_RANGE; }
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    std::lock_guard<std::mutex> lock(ctx->mu);
    cudaStream_t st = user_stream;  // NULL: the legacy default stream
    const uint64_t n = 1ull << L;
    ZK_TRY(ensure_scratch(ctx, 4 * n * 32));
    Fr* buf = (Fr*)ctx->scratch;
    Fr* A = buf + n;
    Fr* B = buf + 2 * n;
    Fr* Cc = buf + 3 * n;
    zkh::Fe g, zinv;
    ZK_TRY(coset_shift(L, g, zinv));
    const CosetTables *to_coset, *from_coset;
    ZK_TRY(get_coset_tables(ctx, L, 2, g, &to_coset));    // n^-1 g^i
    ZK_TRY(get_coset_tables(ctx, L, 1, g, &from_coset));  // n^-1 g^-i
    int launches = 0;
    ZK_TRY(scratch_begin(ctx, st));
    const Fr* ev[3] = {(const Fr*)d_a, (const Fr*)d_b, (const Fr*)d_c};
    Fr* co[3] = {A, B, Cc};
    for (int k = 0; k < 3; k++) {
        FinalOp f1;
        f1.mode = 2;
        f1.tab = to_coset;  // coefficients times n^-1 g^i: the coset shift is fused into the INTT
        ZK_TRY(ntt_core(ctx, st, co[k], ev[k], buf, L, true, nullptr, f1, &launches));
        FinalOp f2;
        if (k == 2) {  // pointwise (A B - C) / (g^n - 1) fused into the last forward permute
            f2.mode = 1;
            std::memcpy(f2.scale.v, zinv.v, 32);
            f2.pa = A;
            f2.pb = B;
        }
        ZK_TRY(ntt_core(ctx, st, co[k], co[k], buf, L, false, nullptr, f2, &launches));
    }
    FinalOp f3;
    f3.mode = 2;
    f3.tab = from_coset;
    ZK_TRY(ntt_core(ctx, st, (Fr*)d_h, Cc, buf, L, true, nullptr, f3, &launches));
    g_ntt_launches = launches;
    return scratch_end(ctx, st);
}

// ------------------------------------------------------------------ allocation-free variant
// zk_ntt_device_noalloc: the same transform with no device allocation at any
// call.  Its working buffer and its tables live in g_ntt_noalloc_scratch, one
// fixed array per device compiled into this library; the tables are
// regenerated on the device at every call, so nothing is cached between
// calls, and every word of the array is written by a call before that call
// reads it (nothing must start at zero).  All calls on one device share the
// array: calls whose work overlaps in time race.
static constexpr int kNoallocMaxLog = ZK_NTT_NOALLOC_MAX_LOG;
static constexpr size_t kNoallocBufElems = (size_t)1 << kNoallocMaxLog;
static constexpr size_t kNoallocTableElems = 4096;  // >= 255 roots + 4 * 2^((L+1)/2) for L <= 18
static_assert(255 + 4 * ((size_t)1 << ((kNoallocMaxLog + 1) / 2)) <= kNoallocTableElems, "noalloc table region too small");

static __device__ __align__(256) Fr g_ntt_noalloc_scratch[kNoallocBufElems + kNoallocTableElems];

struct PowSeg {  // out[offset + k] = start * base^k, k < count
    Fr start, base;
    uint32_t offset, count;
};
struct PowPlan {
    PowSeg seg[12];
    int nseg;
    uint32_t total;  // segments are contiguous: seg[s + 1].offset == seg[s].offset + seg[s].count
};

__global__ void ntt_powers_kernel(Fr* __restrict__ out, PowPlan plan) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < plan.total; i += gridDim.x * blockDim.x) {
        int s = 0;
        while (s + 1 < plan.nseg && i >= plan.seg[s + 1].offset) s++;
        uint32_t k = i - plan.seg[s].offset;
        Fr acc = plan.seg[s].start, b = plan.seg[s].base;
        while (k) {  // square-and-multiply: the canonical Montgomery value equals the host's running product
            if (k & 1) fmul(acc, acc, b);
            k >>= 1;
            if (k) fmul(b, b, b);
        }
        fstore(out + i, acc);
    }
}

struct NoallocDevice {
    std::atomic<bool> ready{false};
    Fr* base = nullptr;  // device address of g_ntt_noalloc_scratch
    int num_sms = 0;
};
static NoallocDevice g_noalloc[64];
static std::mutex g_noalloc_mu;

// One-time set-up per device, with that device current: the array's device
// address, the SM count, and the kernels' attributes (which loads their code).
static int noalloc_setup(int device, NoallocDevice** out) {
    NoallocDevice& d = g_noalloc[device];
    if (d.ready.load(std::memory_order_acquire)) {
        *out = &d;
        return ZK_OK;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!d.ready.load(std::memory_order_relaxed)) {
        int major = 0;
        ZK_TRY_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
        if (major < 10) {
            set_error("device %d has compute capability %d.x; this library is built for sm_100a only", device, major);
            return ZK_ERR_NODEV;
        }
        ZK_TRY_CUDA(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, device));
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_ntt_noalloc_scratch);
        if (e != cudaSuccess || !ptr) {
            set_error("ntt_noalloc: cudaGetSymbolAddress failed on device %d (%s)", device, cudaGetErrorString(e));
            return ZK_ERR_CUDA;
        }
        d.base = (Fr*)ptr;
        for (int r = 1; r <= kMaxLogR; r++)
            ZK_TRY_CUDA(cudaFuncSetAttribute((const void*)pass_fn(r), cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
        cudaFuncAttributes fa;
        ZK_TRY_CUDA(cudaFuncGetAttributes(&fa, (const void*)ntt_permute_kernel));
        ZK_TRY_CUDA(cudaFuncGetAttributes(&fa, (const void*)ntt_powers_kernel));
        d.ready.store(true, std::memory_order_release);
    }
    *out = &d;
    return ZK_OK;
}

static void add_seg(PowPlan& plan, const zkh::Fe& start, const zkh::Fe& base, uint32_t count) {
    PowSeg& s = plan.seg[plan.nseg++];
    std::memcpy(s.start.v, start.v, 32);
    std::memcpy(s.base.v, base.v, 32);
    s.offset = plan.total;
    s.count = count;
    plan.total += count;
}

static int ntt_noalloc_run(int device, cudaStream_t st, void* d_out, const void* d_in, int L, bool inverse, const void* coset_g) {
    if (!d_out || !d_in) { set_error("ntt_noalloc: null pointer"); return ZK_ERR_INVALID; }
    if (L < 0 || L > kNoallocMaxLog) {
        set_error("ntt_noalloc: log_n = %d outside [0, %d] (its fixed buffer holds 2^%d elements)", L, kNoallocMaxLog, kNoallocMaxLog);
        return ZK_ERR_RANGE;
    }
    int count = 0;
    cudaError_t ce = cudaGetDeviceCount(&count);
    if (ce != cudaSuccess || count == 0) {
        set_error("no usable CUDA device (%s)", ce == cudaSuccess ? "device count is 0" : cudaGetErrorString(ce));
        return ZK_ERR_NODEV;
    }
    if (device < 0) ZK_TRY_CUDA(cudaGetDevice(&device));
    if (device >= count || device >= 64) {
        set_error("device %d out of range (%d visible)", device, count);
        return ZK_ERR_INVALID;
    }
    ZK_TRY_CUDA(cudaSetDevice(device));
    NoallocDevice* nd;
    ZK_TRY(noalloc_setup(device, &nd));

    // table region layout: roots (255) | tw_lo | tw_hi | coset lo | coset hi
    Fr* buf = nd->base;
    Fr* tab = nd->base + kNoallocBufElems;
    const zkh::Fe one = zkh::one(zkh::kR);
    const int h = (L + 1) / 2;
    PowPlan plan;
    plan.nseg = 0;
    plan.total = 0;
    NttDirTables T;
    if (L > 0) {
        for (int r = 1; r <= kMaxLogR; r++) add_seg(plan, one, host_root(r, inverse), 1u << (r - 1));
        T.roots = tab;
        T.h = h;
        zkh::Fe w = host_root(L, inverse), wh = w;
        T.tw_lo = tab + plan.total;
        add_seg(plan, one, w, 1u << h);
        for (int i = 0; i < h; i++) zkh::mul(zkh::kR, wh, wh, wh);
        T.tw_hi = tab + plan.total;
        add_seg(plan, one, wh, 1u << (L - h));
    }
    CosetTables cs;
    const CosetTables* pre = nullptr;
    FinalOp fin;
    if (coset_g) {  // the factors of get_coset_tables, kind 0 (forward) or kind 1 (inverse)
        zkh::Fe g, step, start = one;
        std::memcpy(g.v, coset_g, 32);
        step = g;
        if (inverse) {
            zkh::inv(zkh::kR, step, g);
            Fr ninv = n_inverse_dev(L);
            std::memcpy(start.v, ninv.v, 32);
        }
        cs.h = h;
        cs.lo = tab + plan.total;
        add_seg(plan, start, step, 1u << h);
        zkh::Fe sh = step;
        for (int i = 0; i < h; i++) zkh::mul(zkh::kR, sh, sh, sh);
        cs.hi = tab + plan.total;
        add_seg(plan, one, sh, 1u << (L - h));
        if (inverse) {
            fin.mode = 2;
            fin.tab = &cs;
        } else {
            pre = &cs;
        }
    } else if (inverse) {
        fin.mode = 1;
        fin.scale = n_inverse_dev(L);
    }
    int launches = 0;
    if (plan.total) {
        ntt_powers_kernel<<<(plan.total + 255) / 256, 256, 0, st>>>(tab, plan);
        launches++;
    }
    const uint64_t n = 1ull << L;
    Fr* dst = (Fr*)d_out;
    const Fr* src = (const Fr*)d_in;
    if (L == 0) {
        PermPlan none;
        none.P = 0;
        ntt_permute_kernel<<<1, 32, 0, st>>>(src, dst, 0, none, fin.mode, fin.scale, fin.tab ? fin.tab->lo : nullptr,
                                             fin.tab ? fin.tab->hi : nullptr, fin.tab ? fin.tab->h : 0, nullptr, nullptr);
        launches++;
    } else {
        PermPlan pp = make_pass_plan(L);
        int Lp = L;
        const Fr* in = src;
        for (int p = 0; p < pp.P; p++) {
            const int r = pp.r[p];
            const uint64_t M = 1ull << (Lp - r);
            const uint64_t lines = n >> r;
            const int C = M >= 8 ? 8 : (int)std::min<uint64_t>(lines, (uint64_t)std::max(1, kTileElems >> r));
            const size_t smem = ((size_t)(1 << r) * C + (1 << r) / 2 + 1) * sizeof(Fr);
            pass_fn(r)<<<(unsigned)(lines / C), kNttThreads, smem, st>>>(in, buf, L, Lp, C, T.roots, T.tw_lo, T.tw_hi, T.h,
                                                                          (p == 0 && pre) ? pre->lo : nullptr,
                                                                          (p == 0 && pre) ? pre->hi : nullptr, pre ? pre->h : 0);
            launches++;
            in = buf;
            Lp -= r;
        }
        const unsigned pgrid = (unsigned)std::min<uint64_t>((n + 255) / 256, (uint64_t)nd->num_sms * 16);
        ntt_permute_kernel<<<pgrid, 256, 0, st>>>(buf, dst, L, pp, fin.mode, fin.scale, fin.tab ? fin.tab->lo : nullptr,
                                                  fin.tab ? fin.tab->hi : nullptr, fin.tab ? fin.tab->h : 0, nullptr, nullptr);
        launches++;
    }
    ZK_TRY_CUDA(cudaGetLastError());
    g_ntt_launches = launches;
    return ZK_OK;
}

}  // namespace zk

using namespace zk;

extern "C" int zk_ntt_device(int device, void* stream, void* d_out, const void* d_in, int log_n, int inverse, const void* coset_shift) {
    clear_error();
    return ntt_run(device, (cudaStream_t)stream, d_out, d_in, log_n, inverse != 0, coset_shift);
}

extern "C" int zk_compute_h_device(int device, void* stream, void* d_h, const void* d_a, const void* d_b, const void* d_c, int log_n) {
    clear_error();
    return compute_h_run(device, (cudaStream_t)stream, d_h, d_a, d_b, d_c, log_n);
}

// reference-shaped: synchronous on the current device
extern "C" int zk_ntt(void* d_out, const void* d_in, int log_n, int inverse) {
    clear_error();
    if (log_n < 0 || log_n > ZK_REF_NTT_MAX_LOG) {
        set_error("[NTT] Error: log_n=%d exceeds max %d", log_n, ZK_REF_NTT_MAX_LOG);
        return ZK_ERR_RANGE;
    }
    ZK_TRY(ntt_run(-1, nullptr, d_out, d_in, log_n, inverse != 0, nullptr));
    DeviceContext* ctx;
    ZK_TRY(get_context(-1, &ctx));
    ZK_TRY_CUDA(cudaStreamSynchronize(0));
    return ZK_OK;
}

extern "C" int zk_ntt_inplace(void* d_data, int log_n, int inverse) { return zk_ntt(d_data, d_data, log_n, inverse); }

extern "C" int zk_compute_omega(int log_n, int inverse, void* out_fr) {
    clear_error();
    if (!out_fr) return ZK_ERR_INVALID;
    if (log_n < 0 || log_n > ZK_NTT_MAX_LOG) { set_error("compute_omega: log_n = %d out of range", log_n); return ZK_ERR_RANGE; }
    zkh::Fe w = host_root(log_n, inverse != 0);
    std::memcpy(out_fr, w.v, 32);
    return ZK_OK;
}

extern "C" int zk_ntt_device_noalloc(int device, void* stream, void* d_out, const void* d_in, int log_n, int inverse,
                                     const void* coset_shift) {
    clear_error();
    return ntt_noalloc_run(device, (cudaStream_t)stream, d_out, d_in, log_n, inverse != 0, coset_shift);
}

extern "C" int zk_ntt_cross_device(int device, void* stream, void* d_out, const void* d_in, int log_n, int log_parts, int part,
                                   int inverse, int mode, const void* factor_g, int factor_inverse) {
    clear_error();
    return ntt_cross_run(device, (cudaStream_t)stream, d_out, d_in, log_n, log_parts, part, inverse != 0, mode, factor_g,
                         factor_inverse != 0);
}

extern "C" int zk_compute_h_coset_shift(int log_n, void* out_g) {
    clear_error();
    if (!out_g) return ZK_ERR_INVALID;
    if (log_n < 0 || log_n > ZK_NTT_MAX_LOG) { set_error("compute_h: log_n = %d out of range", log_n); return ZK_ERR_RANGE; }
    zkh::Fe g, zinv;
    ZK_TRY(coset_shift(log_n, g, zinv));
    std::memcpy(out_g, g.v, 32);
    return ZK_OK;
}

extern "C" int zk_compute_h_pointwise_device(int device, void* stream, void* d_out, const void* d_a, const void* d_b, const void* d_c,
                                             int log_n, uint64_t count) {
    clear_error();
    if (!d_out || !d_a || !d_b || !d_c) return ZK_ERR_INVALID;
    if (log_n < 0 || log_n > ZK_NTT_MAX_LOG) { set_error("compute_h: log_n = %d out of range", log_n); return ZK_ERR_RANGE; }
    if (count > (1ull << log_n)) { set_error("compute_h: %llu values exceed the 2^%d-point domain", (unsigned long long)count, log_n); return ZK_ERR_RANGE; }
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    zkh::Fe g, zinv;
    ZK_TRY(coset_shift(log_n, g, zinv));
    Fr zi;
    std::memcpy(zi.v, zinv.v, 32);
    const uint64_t n = count;
    if (n == 0) return ZK_OK;
    const unsigned grid = (unsigned)std::min<uint64_t>((n + 255) / 256, (uint64_t)ctx->num_sms * 16);
    h_pointwise_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((Fr*)d_out, (const Fr*)d_a, (const Fr*)d_b, (const Fr*)d_c, n, zi);
    ZK_TRY_CUDA(cudaGetLastError());
    return ZK_OK;
}
