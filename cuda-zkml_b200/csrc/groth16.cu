// groth16.cu -- device-resident Groth16 prover, GPU setup and the proving-key,
// verification-key and proof formats of gdtsitlauri/cuda-zkml.
//
// prove (replaces Groth16Prover::prove, src/prover/groth16.cu:655-920, and the
// host parts of compute_h, :263-390):
//   witness H2D -> sparse matvec A*w, B*w, C*w on the device (the reference does
//   it on the host, :275-294) -> compute_h (7 NTTs, coset shift and pointwise
//   fused, ntt.cu) -> MSMs A, B (G2), L, H, B1 on the device -> on the host:
//     A = alpha1 + sum w_i A_i + r delta1
//     B = beta2  + sum w_i B_i + s delta2
//     C = sum_priv w_i L_i + sum h_j H_j + s A + r (beta1 + sum w_i B1_i)
//   (the reference's convention, :774-844), serialised as the 256-byte proof.
// The proving key and the R1CS stay resident on the device between proofs.
//
// setup (replaces the host loop of Groth16Prover::setup, :446-642): the QAP
// evaluations at tau and the query scalars on the host, then every query point
// k * G by the device fixed-base kernel; the points are canonical, so the key is
// byte-identical to the reference's for the same toxic waste.
#include "prover.hpp"

#include <unistd.h>

#include <atomic>
#include <chrono>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace zk {

// ------------------------------------------------------------------ helpers
static zkh::Fe fr_one() { return zkh::one(zkh::kR); }
static zkh::Fe fr_mul(const zkh::Fe& a, const zkh::Fe& b) { zkh::Fe r; zkh::mul(zkh::kR, r, a, b); return r; }
static zkh::Fe fr_add(const zkh::Fe& a, const zkh::Fe& b) { zkh::Fe r; zkh::add(zkh::kR, r, a, b); return r; }
static zkh::Fe fr_sub(const zkh::Fe& a, const zkh::Fe& b) { zkh::Fe r; zkh::sub(zkh::kR, r, a, b); return r; }
static zkh::Fe fr_inv(const zkh::Fe& a) { zkh::Fe r; zkh::inv(zkh::kR, r, a); return r; }

// primitive 2^L-th root of unity 5^((r-1)/2^L) (src/ntt/ntt.cu:43-106)
static zkh::Fe root_of_unity(int L) {
    uint64_t e[4];
    std::memcpy(e, zkh::kR.m, 32);
    e[0] -= 1;
    for (int s = 0; s < 28; s++)
        for (int i = 0; i < 4; i++) e[i] = (e[i] >> 1) | (i < 3 ? e[i + 1] << 63 : 0);
    uint64_t five[4] = {5, 0, 0, 0};
    zkh::Fe g, w;
    zkh::from_std(zkh::kR, g, five);
    zkh::pow(zkh::kR, w, g, e);
    for (int i = 0; i < 28 - L; i++) w = fr_mul(w, w);
    return w;
}

// batch inversion (Montgomery's trick); zero entries stay zero
static void batch_inverse(std::vector<zkh::Fe>& v) {
    const size_t n = v.size();
    std::vector<zkh::Fe> pre(n);
    zkh::Fe acc = fr_one();
    for (size_t i = 0; i < n; i++) {
        pre[i] = acc;
        if (!zkh::is_zero(v[i])) acc = fr_mul(acc, v[i]);
    }
    zkh::Fe inv = fr_inv(acc);
    for (size_t i = n; i-- > 0;) {
        if (zkh::is_zero(v[i])) continue;
        zkh::Fe t = fr_mul(inv, pre[i]);
        inv = fr_mul(inv, v[i]);
        v[i] = t;
    }
}

template <class F>
static void load_aff(zkh::Xyzz<F>& p, const uint64_t* rec);
template <>
void load_aff<zkh::Fe>(zkh::Xyzz<zkh::Fe>& p, const uint64_t* r) {
    bool z = true;
    for (int i = 0; i < 8; i++) if (r[i]) z = false;
    if (z) { zkh::set_identity(p); return; }
    zkh::Fe x, y;
    std::memcpy(x.v, r, 32);
    std::memcpy(y.v, r + 4, 32);
    zkh::from_affine(p, x, y);
}
template <>
void load_aff<zkh::Fp2>(zkh::Xyzz<zkh::Fp2>& p, const uint64_t* r) {
    bool z = true;
    for (int i = 0; i < 16; i++) if (r[i]) z = false;
    if (z) { zkh::set_identity(p); return; }
    zkh::Fp2 x, y;
    std::memcpy(x.c0.v, r, 32);
    std::memcpy(x.c1.v, r + 4, 32);
    std::memcpy(y.c0.v, r + 8, 32);
    std::memcpy(y.c1.v, r + 12, 32);
    zkh::from_affine(p, x, y);
}
static void store_aff(uint64_t* r, const zkh::Xyzz<zkh::Fe>& p) {
    zkh::Fe x, y;
    zkh::to_affine(x, y, p);
    std::memcpy(r, x.v, 32);
    std::memcpy(r + 4, y.v, 32);
}
static void store_aff(uint64_t* r, const zkh::Xyzz<zkh::Fp2>& p) {
    zkh::Fp2 x, y;
    zkh::to_affine(x, y, p);
    std::memcpy(r, x.c0.v, 32);
    std::memcpy(r + 4, x.c1.v, 32);
    std::memcpy(r + 8, y.c0.v, 32);
    std::memcpy(r + 12, y.c1.v, 32);
}

}  // namespace zk

namespace zk {

static thread_local zk_prove_stats g_prove_stats;

// ------------------------------------------------------------------ kernels
// acc += sum_{j = a, a + step, ... < b} val_j w[col_j], four products per
// Montgomery reduction (a dot product is a sum of products)
__device__ __forceinline__ void row_dot(Fr& acc, const Fr* __restrict__ val, const int32_t* __restrict__ col, const Fr* __restrict__ w,
                                        int a, int b, int step) {
    int j = a;
    for (; j + 3 * step < b; j += 4 * step) {
        Fr v[4], x[4], s;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            fload_nc(v[k], val + j + k * step);
            fload_nc(x[k], w + col[j + k * step]);
        }
        fmulsum_inline<ModR, 4>(s, v, x);
        fadd(acc, acc, s);
    }
    for (; j < b; j += step) {
        Fr v, x;
        fload_nc(v, val + j);
        fload_nc(x, w + col[j]);
        fmul(v, v, x);
        fadd(acc, acc, v);
    }
}

// rows [lo, hi) of M w into out[r - lo]; rows at or beyond `rows` (the
// constraint count) are zero.  Rows with at most kShortRow entries: one thread
// per row; long rows are skipped here and done by r1cs_matvec_long_kernel.
__global__ void r1cs_matvec_short_kernel(const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col, const Fr* __restrict__ val,
                                         const Fr* __restrict__ w, int rows, uint64_t lo, uint64_t hi, Fr* __restrict__ out) {
    for (uint64_t r = lo + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < hi; r += (uint64_t)gridDim.x * blockDim.x) {
        Fr acc;
        fset_zero(acc);
        if (r < (uint64_t)rows) {
            const int a = row_ptr[r], b = row_ptr[r + 1];
            if (b - a <= kShortRow) {
                row_dot(acc, val, col, w, a, b, 1);
            } else {
                continue;  // written by the warp or block kernel
            }
        }
        fstore(out + (r - lo), acc);
    }
}

// one warp per medium row: strided partial sums, then a shuffle tree
__global__ void __launch_bounds__(256) r1cs_matvec_warp_kernel(const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col,
                                                               const Fr* __restrict__ val, const Fr* __restrict__ w,
                                                               const int32_t* __restrict__ rows, size_t count, uint64_t lo,
                                                               Fr* __restrict__ out) {
    const uint32_t lane = threadIdx.x & 31;
    const size_t wid = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (wid >= count) return;  // uniform across the warp
    const int r = rows[wid];
    const int a = row_ptr[r], b = row_ptr[r + 1];
    Fr acc;
    fset_zero(acc);
    row_dot(acc, val, col, w, a + (int)lane, b, 32);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Fr t;
#pragma unroll
        for (int k = 0; k < 8; k++) t.v[k] = __shfl_down_sync(0xffffffffu, acc.v[k], o);
        fadd(acc, acc, t);  // lanes >= 32 - o add their own value again; only lane 0 is kept
    }
    if (lane == 0) fstore(out + (r - lo), acc);
}

// one block per long row: strided partial sums, then a shared-memory tree
__global__ void __launch_bounds__(256) r1cs_matvec_long_kernel(const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col,
                                                               const Fr* __restrict__ val, const Fr* __restrict__ w,
                                                               const int32_t* __restrict__ long_rows, uint64_t lo, Fr* __restrict__ out) {
    __shared__ Fr part[256];
    const int r = long_rows[blockIdx.x];
    const int a = row_ptr[r], b = row_ptr[r + 1];
    Fr acc;
    fset_zero(acc);
    row_dot(acc, val, col, w, a + (int)threadIdx.x, b, (int)blockDim.x);
    part[threadIdx.x] = acc;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if ((int)threadIdx.x < s) {
            Fr t = part[threadIdx.x];
            fadd(t, t, part[threadIdx.x + s]);
            part[threadIdx.x] = t;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) fstore(out + (r - lo), part[0]);
}

// first index i < count with a_i * b_i != c_i (row0 + i is stored), by atomicMin
__global__ void hadamard_check_kernel(const Fr* __restrict__ a, const Fr* __restrict__ b, const Fr* __restrict__ c, uint64_t count,
                                      uint64_t row0, unsigned long long* __restrict__ first_bad) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x) {
        Fr x, y, z;
        fload_nc(x, a + i);
        fload_nc(y, b + i);
        fload_nc(z, c + i);
        fmul(x, x, y);
        uint32_t d = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) d |= x.v[k] ^ z.v[k];  // canonical representatives: equal values, equal words
        if (d) atomicMin(first_bad, (unsigned long long)(row0 + i));
    }
}


// ------------------------------------------------------------------ R1CS upload
static int r1cs_create(int device, int num_constraints, int num_variables, int num_public, const SparseEntry* const* ent,
                       const size_t* nnz, R1cs& R) {
    if (num_constraints < 0 || num_variables <= 0 || num_public < 0 || num_public >= num_variables) {
        set_error("r1cs: invalid sizes (constraints %d, variables %d, public %d)", num_constraints, num_variables, num_public);
        return ZK_ERR_INVALID;
    }
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    R.device = ctx->device;
    R.num_constraints = num_constraints;
    R.m = num_variables;
    R.num_public = num_public;
    // QAP::from_r1cs (groth16.cu:225-242): next power of two, at least 4
    R.n = 1;
    R.log_n = 0;
    while (R.n < (uint64_t)num_constraints) { R.n <<= 1; R.log_n++; }
    if (R.n < 4) { R.n = 4; R.log_n = 2; }
    const int rows = (int)std::min<uint64_t>(R.n, (uint64_t)std::max(num_constraints, 0));
    for (int k = 0; k < 3; k++) {
        Csr& c = R.host[k];
        c.row_ptr.assign((size_t)rows + 1, 0);
        // entries outside the domain or the witness are ignored, as compute_h does (groth16.cu:278-292)
        for (size_t i = 0; i < nnz[k]; i++) {
            const SparseEntry& e = ent[k][i];
            if (e.row >= 0 && e.row < rows && e.col >= 0 && e.col < num_variables) c.row_ptr[(size_t)e.row + 1]++;
        }
        for (int r = 0; r < rows; r++) c.row_ptr[(size_t)r + 1] += c.row_ptr[r];
        const size_t total = (size_t)c.row_ptr[rows];
        c.col.resize(total);
        c.val.resize(total);
        std::vector<int32_t> cur(c.row_ptr.begin(), c.row_ptr.end() - 1);
        for (size_t i = 0; i < nnz[k]; i++) {
            const SparseEntry& e = ent[k][i];
            if (e.row >= 0 && e.row < rows && e.col >= 0 && e.col < num_variables) {
                const int32_t p = cur[e.row]++;
                c.col[p] = e.col;
                std::memcpy(c.val[p].v, e.v, 32);
            }
        }
        c.mid_rows.clear();
        c.long_rows.clear();
        for (int r = 0; r < rows; r++) {
            const int32_t len = c.row_ptr[(size_t)r + 1] - c.row_ptr[r];
            if (len > kMidRow) c.long_rows.push_back(r);
            else if (len > kShortRow) c.mid_rows.push_back(r);
        }
        R.nnz[k] = total;
        ZK_TRY_CUDA(cudaMalloc(&R.d_row_ptr[k], c.row_ptr.size() * 4));
        ZK_TRY_CUDA(cudaMemcpy(R.d_row_ptr[k], c.row_ptr.data(), c.row_ptr.size() * 4, cudaMemcpyHostToDevice));
        ZK_TRY_CUDA(cudaMalloc(&R.d_col[k], std::max<size_t>(total, 1) * 4));
        ZK_TRY_CUDA(cudaMemcpy(R.d_col[k], c.col.data(), total * 4, cudaMemcpyHostToDevice));
        ZK_TRY_CUDA(cudaMalloc(&R.d_val[k], std::max<size_t>(total, 1) * 32));
        ZK_TRY_CUDA(cudaMemcpy(R.d_val[k], c.val.data(), total * 32, cudaMemcpyHostToDevice));
        ZK_TRY_CUDA(cudaMalloc(&R.d_mid[k], std::max<size_t>(c.mid_rows.size(), 1) * 4));
        ZK_TRY_CUDA(cudaMemcpy(R.d_mid[k], c.mid_rows.data(), c.mid_rows.size() * 4, cudaMemcpyHostToDevice));
        ZK_TRY_CUDA(cudaMalloc(&R.d_long[k], std::max<size_t>(c.long_rows.size(), 1) * 4));
        ZK_TRY_CUDA(cudaMemcpy(R.d_long[k], c.long_rows.data(), c.long_rows.size() * 4, cudaMemcpyHostToDevice));
    }
    return ZK_OK;
}

// rows [lo, hi) of A w, B w, C w into out3 (three vectors of hi - lo elements)
int r1cs_matvec_rows(const R1cs& R, cudaStream_t st, const Fr* w, uint64_t lo, uint64_t hi, Fr* out3, int num_sms) {
    const int rows = (int)std::min<uint64_t>(R.n, (uint64_t)R.num_constraints);
    const uint64_t len = hi - lo;
    if (len == 0) return ZK_OK;
    for (int k = 0; k < 3; k++) {
        Fr* out = out3 + (size_t)k * len;
        const unsigned grid = (unsigned)std::min<uint64_t>((len + 255) / 256, (uint64_t)num_sms * 16);
        r1cs_matvec_short_kernel<<<grid, 256, 0, st>>>(R.d_row_ptr[k], R.d_col[k], R.d_val[k], w, rows, lo, hi, out);
        // medium and long rows inside [lo, hi): contiguous runs of the ascending lists
        const std::vector<int32_t>& mr = R.host[k].mid_rows;
        const size_t ma = std::lower_bound(mr.begin(), mr.end(), (int64_t)lo) - mr.begin();
        const size_t mb = std::lower_bound(mr.begin(), mr.end(), (int64_t)hi) - mr.begin();
        if (mb > ma)
            r1cs_matvec_warp_kernel<<<(unsigned)((mb - ma + 7) / 8), 256, 0, st>>>(R.d_row_ptr[k], R.d_col[k], R.d_val[k], w,
                                                                                  R.d_mid[k] + ma, mb - ma, lo, out);
        const std::vector<int32_t>& lr = R.host[k].long_rows;
        const size_t a = std::lower_bound(lr.begin(), lr.end(), (int64_t)lo) - lr.begin();
        const size_t b = std::lower_bound(lr.begin(), lr.end(), (int64_t)hi) - lr.begin();
        if (b > a)
            r1cs_matvec_long_kernel<<<(unsigned)(b - a), 256, 0, st>>>(R.d_row_ptr[k], R.d_col[k], R.d_val[k], w, R.d_long[k] + a, lo,
                                                                      out);
    }
    ZK_TRY_CUDA(cudaGetLastError());
    return ZK_OK;
}

static int r1cs_matvec(const R1cs& R, cudaStream_t st, const Fr* w, Fr* out3, int num_sms) {
    return r1cs_matvec_rows(R, st, w, 0, R.n, out3, num_sms);
}

// The reference's verify_witness (src/prover/circuit.cuh:93-124): every
// constraint row r satisfies (A w)_r (B w)_r = (C w)_r.  Enqueues the check of
// rows [row0, row0 + count) on `st`; *first_bad (device) must start at
// 0xff..ff and ends as the first failing row, if any.
void enqueue_hadamard_check(cudaStream_t st, const Fr* a, const Fr* b, const Fr* c, uint64_t count, uint64_t row0,
                                   unsigned long long* first_bad, int num_sms) {
    if (!count) return;
    const unsigned grid = (unsigned)std::min<uint64_t>((count + 255) / 256, (uint64_t)num_sms * 16);
    hadamard_check_kernel<<<grid, 256, 0, st>>>(a, b, c, count, row0, first_bad);
}

bool witness_check_enabled() {
    // ZKML_SKIP_WITNESS_CHECK=1 turns the check off, as in Groth16Prover::prove (groth16.cu:691-697)
    const char* e = std::getenv("ZKML_SKIP_WITNESS_CHECK");
    return !(e && std::strcmp(e, "1") == 0);
}

// ------------------------------------------------------------------ setup
// QAP evaluations at tau (groth16.cu:97-189):
//   L_j(tau) = (tau^n - 1) w^j / (n (tau - w^j)),  X_at[col] += value * L_row(tau)
static void qap_at_tau(const R1cs& R, const zkh::Fe& tau, std::vector<zkh::Fe> at[3], zkh::Fe& vanish) {
    const uint64_t n = R.n;
    const zkh::Fe w = root_of_unity(R.log_n);
    zkh::Fe tn = tau;
    for (int i = 0; i < R.log_n; i++) tn = fr_mul(tn, tn);
    vanish = fr_sub(tn, fr_one());
    uint64_t s2[4] = {2, 0, 0, 0};
    zkh::Fe two;
    zkh::from_std(zkh::kR, two, s2);
    zkh::Fe half = fr_inv(two), ninv = fr_one();
    for (int i = 0; i < R.log_n; i++) ninv = fr_mul(ninv, half);
    std::vector<zkh::Fe> den(n), lag(n);
    zkh::Fe wj = fr_one();
    for (uint64_t j = 0; j < n; j++) {
        den[j] = fr_sub(tau, wj);
        lag[j] = fr_mul(fr_mul(vanish, wj), ninv);
        wj = fr_mul(wj, w);
    }
    batch_inverse(den);
    for (uint64_t j = 0; j < n; j++) lag[j] = fr_mul(lag[j], den[j]);
    for (int k = 0; k < 3; k++) {
        at[k].assign((size_t)R.m, zkh::zero());
        const Csr& c = R.host[k];
        const int rows = (int)c.row_ptr.size() - 1;
        for (int r = 0; r < rows; r++)
            for (int p = c.row_ptr[r]; p < c.row_ptr[(size_t)r + 1]; p++) at[k][c.col[p]] = fr_add(at[k][c.col[p]], fr_mul(c.val[p], lag[r]));
    }
}

static int setup(const R1cs& R, const zkh::Fe toxic[5], zk_groth16_pk* pk) {
    const zkh::Fe tau = toxic[0], alpha = toxic[1], beta = toxic[2], gamma = toxic[3], delta = toxic[4];
    const int m = R.m, pub = R.num_public;
    const int l = std::max(0, m - pub - 1);
    const uint64_t n = R.n;
    std::vector<zkh::Fe> at[3];
    zkh::Fe vanish;
    qap_at_tau(R, tau, at, vanish);
    const zkh::Fe dinv = fr_inv(delta), ginv = fr_inv(gamma);
    // G1 scalars: A[m] | B[m] | L[l] | H[n] | IC[pub+1] | alpha, beta, delta
    const size_t nG1 = 2 * (size_t)m + l + n + (size_t)pub + 1 + 3;
    std::vector<zkh::Fe> s1(nG1);
    size_t o = 0;
    for (int i = 0; i < m; i++) s1[o++] = at[0][i];
    for (int i = 0; i < m; i++) s1[o++] = at[1][i];
    auto lc = [&](int i) { return fr_add(fr_add(fr_mul(beta, at[0][i]), fr_mul(alpha, at[1][i])), at[2][i]); };
    for (int i = 0; i < l; i++) s1[o++] = fr_mul(lc(i + 1 + pub), dinv);
    zkh::Fe tp = fr_mul(vanish, dinv);
    for (uint64_t i = 0; i < n; i++) { s1[o++] = tp; tp = fr_mul(tp, tau); }
    for (int i = 0; i <= pub; i++) s1[o++] = fr_mul(lc(i), ginv);
    s1[o++] = alpha;
    s1[o++] = beta;
    s1[o++] = delta;
    // G2 scalars: B[m] | beta, gamma, delta, tau, 1
    std::vector<zkh::Fe> s2(at[1]);
    s2.push_back(beta);
    s2.push_back(gamma);
    s2.push_back(delta);
    s2.push_back(tau);
    s2.push_back(fr_one());

    DeviceContext* ctx;
    ZK_TRY(get_context(R.device, &ctx));
    // freed on every exit path; the two point arrays pass to the key on success
    DeviceBuffer sc_buf, g1_buf, g2_buf;
    ZK_TRY_CUDA(sc_buf.alloc(std::max(nG1, s2.size()) * 32));
    ZK_TRY_CUDA(g1_buf.alloc(nG1 * 64));
    ZK_TRY_CUDA(g2_buf.alloc(s2.size() * 128));
    Fr* d_sc = (Fr*)sc_buf.p;
    uint8_t* g1_all = (uint8_t*)g1_buf.p;
    uint8_t* g2_all = (uint8_t*)g2_buf.p;
    ZK_TRY_CUDA(cudaMemcpy(d_sc, s1.data(), nG1 * 32, cudaMemcpyHostToDevice));
    ZK_TRY(zk_g1_fixed_base_device(R.device, nullptr, g1_all, d_sc, nG1));
    ZK_TRY_CUDA(cudaDeviceSynchronize());
    ZK_TRY_CUDA(cudaMemcpy(d_sc, s2.data(), s2.size() * 32, cudaMemcpyHostToDevice));
    ZK_TRY(zk_g2_fixed_base_device(R.device, nullptr, g2_all, d_sc, s2.size()));
    ZK_TRY_CUDA(cudaDeviceSynchronize());
    std::vector<uint64_t> t1((size_t)(pub + 1 + 3) * 8);
    const size_t tail1 = 2 * (size_t)m + l + n;
    ZK_TRY_CUDA(cudaMemcpy(t1.data(), g1_all + tail1 * 64, t1.size() * 8, cudaMemcpyDeviceToHost));
    std::vector<uint64_t> t2(5 * 16);
    ZK_TRY_CUDA(cudaMemcpy(t2.data(), g2_all + (size_t)m * 128, t2.size() * 8, cudaMemcpyDeviceToHost));

    pk->device = R.device;
    pk->num_constraints = (int)n;
    pk->m = m;
    pk->num_public = pub;
    pk->l = l;
    pk->n_h = (int)n;
    pk->g1 = (uint8_t*)g1_buf.release();  // A | B1 | L | H | IC | alpha beta delta (the tail copied out above)
    pk->g2 = (uint8_t*)g2_buf.release();  // B2 | beta gamma delta tau G2
    pk->ic.assign(t1.begin(), t1.begin() + (size_t)(pub + 1) * 8);
    std::memcpy(pk->alpha1, &t1[(size_t)(pub + 1) * 8], 64);
    std::memcpy(pk->beta1, &t1[(size_t)(pub + 2) * 8], 64);
    std::memcpy(pk->delta1, &t1[(size_t)(pub + 3) * 8], 64);
    std::memcpy(pk->beta2, &t2[0], 128);
    std::memcpy(pk->gamma2, &t2[16], 128);
    std::memcpy(pk->delta2, &t2[32], 128);
    std::memcpy(pk->tau2, &t2[48], 128);
    std::memcpy(pk->g2gen, &t2[64], 128);
    return ZK_OK;
}

static int ensure_prover_buffers(zk_groth16_pk* pk, uint64_t n, int m) {
    if (pk->n_buf >= n && pk->w) return ZK_OK;
    if (pk->w) cudaFree(pk->w);
    if (pk->abc) cudaFree(pk->abc);
    if (pk->h) cudaFree(pk->h);
    ZK_TRY_CUDA(cudaMalloc(&pk->w, (size_t)std::max<uint64_t>(m, 1) * 32));
    ZK_TRY_CUDA(cudaMalloc(&pk->abc, 3 * n * 32));
    ZK_TRY_CUDA(cudaMalloc(&pk->h, n * 32));
    if (!pk->d_bad) ZK_TRY_CUDA(cudaMalloc(&pk->d_bad, sizeof(unsigned long long)));
    if (!pk->h_bad) ZK_TRY_CUDA(cudaMallocHost(&pk->h_bad, sizeof(unsigned long long)));
    pk->n_buf = n;
    return ZK_OK;
}

// k * P from the table tab[i] = 2^i P: one addition per set bit of k
template <class F>
static void fixed_mul(zkh::Xyzz<F>& out, const std::vector<zkh::Xyzz<F>>& tab, const uint64_t k_std[4]) {
    zkh::set_identity(out);
    for (int bit = 0; bit < 256; bit++)
        if ((k_std[bit >> 6] >> (bit & 63)) & 1) zkh::add(out, tab[bit]);
}

template <class F>
static void build_pow2(std::vector<zkh::Xyzz<F>>& tab, const uint64_t* base) {
    zkh::Xyzz<F> p, d;
    load_aff(p, base);
    tab.resize(256);
    for (int i = 0; i < 256; i++) {
        tab[i] = p;
        zkh::dbl(d, p);
        p = d;
    }
}

// Proof points from the five MSM sums (groth16.cu:774-844):
//   A = alpha1 + sum_A + r delta1
//   B = beta2 + sum_B2 + s delta2
//   C = sum_L + sum_H + s A + r (beta1 + sum_B1)
// (the reference folds r s delta1 into s A, with A the affine proof point)
static void assemble_xyzz(const zk_groth16_pk* pk, const zkh::Fe& r, const zkh::Fe& s, const zkh::Xyzz<zkh::Fe>& a_msm,
                          const zkh::Xyzz<zkh::Fp2>& b_msm, const zkh::Xyzz<zkh::Fe>& l_msm, const zkh::Xyzz<zkh::Fe>& h_msm,
                          const zkh::Xyzz<zkh::Fe>& b1_msm, uint64_t outA[8], uint64_t outB[16], uint64_t outC[8]) {
    uint64_t rs[4], ss[4];
    zkh::to_std(zkh::kR, rs, r);
    zkh::to_std(zkh::kR, ss, s);
    using P1 = zkh::Xyzz<zkh::Fe>;
    using P2 = zkh::Xyzz<zkh::Fp2>;
    {
        std::lock_guard<std::mutex> lock(pk->tab_mu);
        if (pk->d1_pow.empty()) build_pow2(pk->d1_pow, pk->delta1);
        if (pk->d2_pow.empty()) build_pow2(pk->d2_pow, pk->delta2);
    }
    P1 A, t1;
    load_aff(A, pk->alpha1);
    zkh::add(A, a_msm);
    fixed_mul(t1, pk->d1_pow, rs);
    zkh::add(A, t1);
    store_aff(outA, A);
    P2 Bp, t2;
    load_aff(Bp, pk->beta2);
    zkh::add(Bp, b_msm);
    fixed_mul(t2, pk->d2_pow, ss);
    zkh::add(Bp, t2);
    store_aff(outB, Bp);
    P1 Cp = l_msm, Aaff, b1;
    zkh::add(Cp, h_msm);
    load_aff(Aaff, outA);          // s * A uses the affine proof point A
    zkh::smul(t1, Aaff, ss);
    zkh::add(Cp, t1);
    load_aff(b1, pk->beta1);
    zkh::add(b1, b1_msm);
    zkh::smul(t1, b1, rs);
    zkh::add(Cp, t1);
    store_aff(outC, Cp);
}

static void assemble(const zk_groth16_pk* pk, const zkh::Fe& r, const zkh::Fe& s, const uint64_t a_msm[8], const uint64_t b_msm[16],
                     const uint64_t l_msm[8], const uint64_t h_msm[8], const uint64_t b1_msm[8], uint64_t outA[8], uint64_t outB[16],
                     uint64_t outC[8]) {
    zkh::Xyzz<zkh::Fe> a, l, h, b1;
    zkh::Xyzz<zkh::Fp2> b;
    load_aff(a, a_msm);
    load_aff(b, b_msm);
    load_aff(l, l_msm);
    load_aff(h, h_msm);
    load_aff(b1, b1_msm);
    assemble_xyzz(pk, r, s, a, b, l, h, b1, outA, outB, outC);
}

// The H MSM of every proof runs over the same bases (the key's H query) with
// uniform 254-bit scalars (h's coefficients): precomputed window tables let all
// its windows share one bucket set and one reduce (msm.cu, msm_tables_run).
// Below kHTablesMin points the plain MSM is as fast.
static constexpr int kHTablesMin = 1 << 16;

// Starts the table build on the key's table stream, once (caller holds h_mu).
// The build's blocks are short (one launch per table entry), and a proof's
// critical path runs at the highest stream priority, so a proof beside the
// build gets SMs as the build's blocks retire.
// optional: a start on behalf of a proof or an H MSM, for which the tables are
// an optimisation: without device memory for them the plain MSM goes on serving
// (and no later call tries again); zk_groth16_precompute asks for them outright.
static int start_h_tables_locked(zk_groth16_pk* pk, bool optional) {
    if (pk->h_tab || pk->h_tab_pending || pk->n_h < kHTablesMin || (optional && pk->h_tab_off)) return ZK_OK;
    int c, W;
    g1_window_tables_shape((size_t)pk->n_h, &c, &W);
    if ((size_t)W * pk->n_h > 0x7fffffffull) return ZK_OK;  // keys index 32 bits: the plain MSM runs in passes
    if (!pk->h_tab_stream) {
        ZK_TRY_CUDA(cudaStreamCreateWithFlags(&pk->h_tab_stream, cudaStreamNonBlocking));
        ZK_TRY_CUDA(cudaEventCreateWithFlags(&pk->h_tab_done, cudaEventDisableTiming));
    }
    DeviceBuffer tab;
    const cudaError_t ae = tab.alloc((size_t)W * pk->n_h * 64);
    if (ae != cudaSuccess) {
        cudaGetLastError();  // an allocation failure is not sticky; clear it for the next call
        if (optional) {
            pk->h_tab_off = true;
            return ZK_OK;
        }
        set_error("H-query window tables (%zu bytes): %s", (size_t)W * pk->n_h * 64, cudaGetErrorString(ae));
        return ae == cudaErrorMemoryAllocation ? ZK_ERR_NOMEM : ZK_ERR_CUDA;
    }
    const uint8_t* hq = pk->g1 + (2 * (size_t)pk->m + pk->l) * 64;
    ZK_TRY(g1_window_tables_build(pk->device, pk->h_tab_stream, hq, (size_t)pk->n_h, c, W, tab.p));
    ZK_TRY_CUDA(cudaEventRecord(pk->h_tab_done, pk->h_tab_stream));
    pk->h_tab_pending = (uint8_t*)tab.release();
    pk->h_pc = c;
    pk->h_pW = W;
    return ZK_OK;
}

// Publishes a finished build (caller holds h_mu); with `wait`, waits for it.
static int publish_h_tables_locked(zk_groth16_pk* pk, bool wait) {
    if (!pk->h_tab_pending) return ZK_OK;
    const cudaError_t q = wait ? cudaEventSynchronize(pk->h_tab_done) : cudaEventQuery(pk->h_tab_done);
    if (q == cudaErrorNotReady) return ZK_OK;
    if (q != cudaSuccess) {
        cudaFree(pk->h_tab_pending);
        pk->h_tab_pending = nullptr;
        set_error("H-query window tables: %s", cudaGetErrorString(q));
        return ZK_ERR_CUDA;
    }
    pk->h_tab = pk->h_tab_pending;
    pk->h_c = pk->h_pc;
    pk->h_W = pk->h_pW;
    pk->h_tab_pending = nullptr;
    return ZK_OK;
}

// The tables, built now if need be (zk_groth16_precompute).
static int ensure_h_tables(zk_groth16_pk* pk) {
    std::lock_guard<std::mutex> lock(pk->h_mu);
    ZK_TRY(start_h_tables_locked(pk, false));
    return publish_h_tables_locked(pk, true);
}

// sum_{i in [lo, hi)} h_i H_i; d_h holds all n_h coefficients.  The tables are
// shaped for the whole query: on a slice under 3/4 of it (a rank's share of a
// split proof) their fixed bucket reduction and wider gathers cost more than a
// plain MSM sized to the slice (measured at half the query: 10.3 vs 9.9 ms).
// Until the tables are built (a build started by the first such call runs on
// its own stream beside the proofs) the plain MSM serves.
// start_build: a call without tables starts their build (a proof starts it
// after its own work instead, so that its buffers grow before the build runs).
static int h_msm(zk_groth16_pk* pk, cudaStream_t st, const Fr* d_h, size_t lo, size_t hi, uint64_t out[8], bool start_build) {
    if ((hi - lo) * 4 >= (size_t)pk->n_h * 3) {
        uint8_t* tab;
        int c, W;
        {
            std::lock_guard<std::mutex> lock(pk->h_mu);
            if (start_build) ZK_TRY(start_h_tables_locked(pk, true));
            ZK_TRY(publish_h_tables_locked(pk, false));
            tab = pk->h_tab;
            c = pk->h_c;
            W = pk->h_W;
        }
        if (tab) return g1_window_tables_msm(pk->device, st, tab, (size_t)pk->n_h, c, W, lo, hi, d_h + lo, out);
    }
    const uint8_t* hq = pk->g1 + (2 * (size_t)pk->m + pk->l) * 64;
    return zk_msm_g1_device(pk->device, st, hq + lo * 64, d_h + lo, hi - lo, out);
}

// One part's share of the H MSM of a proof split over N = 2^log_parts parts,
// its coefficients in the "blocks" layout of the split transforms (local
// k q + v is global k m + part q + v, m = n / N, q = m / N).  The part's H
// points are gathered once into that order (points at or beyond n_h stay the
// identity, all-zero), with window tables over them from 2^16 points when
// the query covers the whole domain.
int h_msm_blocks(zk_groth16_pk* pk, cudaStream_t st, const Fr* d_h_part, int log_parts, int part, uint64_t out[8]) {
    const uint64_t n = (uint64_t)pk->num_constraints;
    if (log_parts < 0 || log_parts > 3 || (n >> (2 * log_parts)) == 0 || part < 0 || part >= (1 << log_parts)) {
        set_error("H MSM blocks: %d parts of a %llu-point domain, part %d out of range", 1 << log_parts, (unsigned long long)n, part);
        return ZK_ERR_RANGE;
    }
    const uint64_t m = n >> log_parts, q = m >> log_parts;
    zk_groth16_pk::HBlocks hb;
    {
        std::lock_guard<std::mutex> lock(pk->h_mu);
        auto it = pk->hb.find({log_parts, part});
        if (it != pk->hb.end()) {
            hb = it->second;
        } else {
            int rc = ZK_OK;
            if (cudaMalloc(&hb.pts, m * 64) != cudaSuccess) rc = ZK_ERR_CUDA;
            if (rc == ZK_OK && cudaMemsetAsync(hb.pts, 0, m * 64, st) != cudaSuccess) rc = ZK_ERR_CUDA;
            const uint8_t* hq = pk->g1 + (2 * (size_t)pk->m + pk->l) * 64;
            for (uint64_t k = 0; rc == ZK_OK && k < (1ull << log_parts); k++) {
                const uint64_t g0 = k * m + (uint64_t)part * q;
                if (g0 >= (uint64_t)pk->n_h) continue;
                const uint64_t cnt = std::min<uint64_t>(q, (uint64_t)pk->n_h - g0);
                if (cudaMemcpyAsync(hb.pts + k * q * 64, hq + g0 * 64, cnt * 64, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
                    rc = ZK_ERR_CUDA;
            }
            // tables need every base on the curve: none when identities fill missing points
            if (rc == ZK_OK && m >= (uint64_t)kHTablesMin && (uint64_t)pk->n_h >= n) {
                g1_window_tables_shape(m, &hb.c, &hb.W);
                if ((size_t)hb.W * m <= 0x7fffffffull) {  // keys index 32 bits: else the plain MSM, in passes
                    // the tables are an optimisation: without room for them the plain MSM serves
                    if (cudaMalloc(&hb.tab, (size_t)hb.W * m * 64) != cudaSuccess) {
                        cudaGetLastError();
                        hb.tab = nullptr;
                    }
                    if (hb.tab) rc = g1_window_tables_build(pk->device, st, hb.pts, m, hb.c, hb.W, hb.tab);
                }
            }
            if (rc == ZK_OK && cudaStreamSynchronize(st) != cudaSuccess) rc = ZK_ERR_CUDA;
            if (rc != ZK_OK) {
                if (rc == ZK_ERR_CUDA) set_error("H MSM blocks: %s", cudaGetErrorString(cudaGetLastError()));
                cudaFree(hb.pts);
                cudaFree(hb.tab);
                return rc;
            }
            pk->hb[{log_parts, part}] = hb;
        }
    }
    if (hb.tab) return g1_window_tables_msm(pk->device, st, hb.tab, m, hb.c, hb.W, 0, m, d_h_part, out);
    return zk_msm_g1_device(pk->device, st, hb.pts, d_h_part, m, out);
}

// The MSMs of a proof whose scalars are the witness (groth16.cu:776-827), over
// the witness slice [lo, hi): A, B (G2) and B1 over its points [lo, hi), L over
// the private part of the slice (L_j pairs with w_{1 + pub + j}).  One
// histogram and one counting sort serve the four.  *all_ms: device time.
int witness_msms(zk_groth16_pk* pk, DeviceContext* ctx, cudaStream_t st, const Fr* d_w, size_t lo, size_t hi, uint64_t a[8], uint64_t b[16],
                        uint64_t b1[8], uint64_t l[8], float set_ms[4], float* all_ms) {
    const size_t m = (size_t)pk->m, pub = (size_t)pk->num_public;
    const size_t num_priv = (size_t)std::max(0, std::min(pk->l, pk->m - 1 - pk->num_public));
    if (lo > hi || hi > m) {
        set_error("witness MSMs: slice [%zu, %zu) outside the %zu-entry witness", lo, hi, m);
        return ZK_ERR_RANGE;
    }
    // L's scalars w[1 + pub, 1 + pub + num_priv) inside the slice, as local indices
    const size_t l_lo = std::max(lo, 1 + pub), l_hi = std::min(hi, 1 + pub + num_priv);
    const bool has_l = l_hi > l_lo;
    const int sets = has_l ? 4 : 3;
    const void* pts[4] = {pk->g1 + lo * 64, pk->g2 + lo * 128, pk->g1 + (m + lo) * 64,
                          pk->g1 + (2 * m + (has_l ? l_lo - 1 - pub : 0)) * 64};
    const int g2[4] = {0, 1, 0, 0};
    const uint32_t range[8] = {0, 0xffffffffu, 0, 0xffffffffu, 0, 0xffffffffu, (uint32_t)(has_l ? l_lo - lo : 0),
                               (uint32_t)(has_l ? l_hi - lo : 0)};
    std::memset(l, 0, 64);
    uint64_t* outs[4] = {a, b, b1, l};
    ZK_TRY_CUDA(cudaSetDevice(ctx->device));  // the events below belong to the context's device
    ScopedEvent s0, s1;
    ZK_TRY_CUDA(cudaEventCreate(&s0.e));
    ZK_TRY_CUDA(cudaEventCreate(&s1.e));
    ZK_TRY_CUDA(cudaEventRecord(s0.e, st));
    ZK_TRY(msm_shared_scalars_run(ctx, st, d_w + lo, hi - lo, sets, pts, g2, range, outs, set_ms));
    ZK_TRY_CUDA(cudaEventRecord(s1.e, st));
    ZK_TRY_CUDA(cudaEventSynchronize(s1.e));
    cudaEventElapsedTime(all_ms, s0.e, s1.e);
    return ZK_OK;
}

// The key's private device context of the witness MSMs (created on first use).
int ensure_witness_context(zk_groth16_pk* pk) {
    std::lock_guard<std::mutex> lock(pk->h_mu);
    if (!pk->wctx) ZK_TRY(create_context(pk->device, &pk->wctx));
    return ZK_OK;
}

// ------------------------------------------------------------------ prove
static int prove(zk_groth16_pk* pk, const R1cs& R, cudaStream_t st, const void* h_witness, const zkh::Fe& r, const zkh::Fe& s,
                 uint64_t outA[8], uint64_t outB[16], uint64_t outC[8]) {
    zk_prove_stats& stats = g_prove_stats;
    std::memset(&stats, 0, sizeof stats);
    if (R.m != pk->m || R.num_public != pk->num_public || (uint64_t)pk->num_constraints != R.n) {
        set_error("prove: proving key (m %d, public %d, n %d) does not match the circuit (m %d, public %d, n %llu)", pk->m,
                  pk->num_public, pk->num_constraints, R.m, R.num_public, (unsigned long long)R.n);
        return ZK_ERR_INVALID;
    }
    DeviceContext* ctx;
    ZK_TRY(get_context(pk->device, &ctx));
    const uint64_t n = R.n;
    const int m = R.m, pub = R.num_public;
    ZK_TRY(ensure_prover_buffers(pk, n, m));
    ZK_TRY(ensure_witness_context(pk));
    ScopedEvent evs[5];
    for (auto& e : evs) ZK_TRY_CUDA(cudaEventCreate(&e.e));
    cudaEvent_t ev[5] = {evs[0].e, evs[1].e, evs[2].e, evs[3].e, evs[4].e};
    // The matvec, compute_h and the H MSM run on a stream of the highest
    // priority, ordered after the caller's stream and before its later work, so
    // that the witness MSMs beside them take what they leave (measured: 29.10 ->
    // 28.80 ms at config 5).  ZK_PROVE_PRIORITY=0 keeps them on the caller's stream.
    const cudaStream_t user_st = st;
    const char* pe = getenv("ZK_PROVE_PRIORITY");
    if (!(pe && atoi(pe) == 0)) {
        if (!pk->prio_stream) {
            int least = 0, greatest = 0;
            ZK_TRY_CUDA(cudaDeviceGetStreamPriorityRange(&least, &greatest));
            ZK_TRY_CUDA(cudaStreamCreateWithPriority(&pk->prio_stream, cudaStreamNonBlocking, greatest));
        }
        ZK_TRY_CUDA(cudaEventRecord(ev[3], user_st));
        ZK_TRY_CUDA(cudaStreamWaitEvent(pk->prio_stream, ev[3], 0));
        st = pk->prio_stream;
    }
    ZK_TRY_CUDA(cudaEventRecord(ev[0], st));
    ZK_TRY_CUDA(cudaMemcpyAsync(pk->w, h_witness, (size_t)m * 32, cudaMemcpyHostToDevice, st));
    ZK_TRY_CUDA(cudaEventRecord(ev[4], st));

    // A, B (G2), B1 and L need only the witness: a worker thread runs them on
    // the key's private context as soon as the witness lands, beside the
    // matvec, compute_h and the H MSM on `st`.  Over a witness (mostly 0/1
    // range-check bits) their bucket fixups and reductions are chains of
    // dependent point additions over few, very full buckets that leave most
    // SMs idle; the NTTs and the H MSM fill them.  One counting sort of the
    // witness serves the four.
    uint64_t a_msm[8], b1_msm[8], l_msm[8] = {0}, h_msm_out[8] = {0}, b_msm[16];
    float set_ms[4] = {0, 0, 0, 0}, wit_all = 0;
    int wit_rc = ZK_OK;
    std::string wit_err;
    struct Joiner {
        std::thread t;
        ~Joiner() {
            if (t.joinable()) t.join();
        }
    } worker;  // joined on every return path, before the results above go out of scope
    DeviceContext* wctx = pk->wctx;
    ZK_TRY_CUDA(cudaStreamWaitEvent(wctx->stream, ev[4], 0));
    worker.t = std::thread([&, wctx]() {
        // a new thread starts on device 0: everything it creates must live on the key's device
        if (cudaSetDevice(wctx->device) != cudaSuccess) {
            wit_rc = ZK_ERR_CUDA;
            wit_err = std::string("witness MSMs: cudaSetDevice: ") + cudaGetErrorString(cudaGetLastError());
            return;
        }
        wit_rc = witness_msms(pk, wctx, wctx->stream, pk->w, 0, (size_t)m, a_msm, b_msm, b1_msm, l_msm, set_ms, &wit_all);
        if (wit_rc != ZK_OK) wit_err = zk_last_error();
    });

    ZK_TRY(r1cs_matvec(R, st, pk->w, pk->abc, ctx->num_sms));
    const bool check = witness_check_enabled();
    if (check) {
        ZK_TRY_CUDA(cudaMemsetAsync(pk->d_bad, 0xff, sizeof(unsigned long long), st));
        enqueue_hadamard_check(st, pk->abc, pk->abc + n, pk->abc + 2 * n, std::min<uint64_t>(n, (uint64_t)R.num_constraints), 0,
                               pk->d_bad, ctx->num_sms);
        ZK_TRY_CUDA(cudaMemcpyAsync(pk->h_bad, pk->d_bad, sizeof(unsigned long long), cudaMemcpyDeviceToHost, st));
    }
    ZK_TRY_CUDA(cudaEventRecord(ev[1], st));
    ZK_TRY(zk_compute_h_device(pk->device, st, pk->h, pk->abc, pk->abc + n, pk->abc + 2 * n, R.log_n));
    ZK_TRY_CUDA(cudaEventRecord(ev[2], st));
    ZK_TRY_CUDA(cudaEventSynchronize(ev[2]));
    if (check && *pk->h_bad != ~0ull) {
        set_error("[Prove] Witness does not satisfy R1CS constraints (constraint %llu failed)", *pk->h_bad);
        return ZK_ERR_INVALID;
    }
    float ms;
    cudaEventElapsedTime(&ms, ev[0], ev[1]);
    stats.matvec_ms = ms;
    cudaEventElapsedTime(&ms, ev[1], ev[2]);
    stats.compute_h_ms = ms;

    zk_msm_stats ms_st;
    const int n_h = std::min<int>((int)n, pk->n_h);
    if (n_h > 0) {
        ZK_TRY(h_msm(pk, st, pk->h, 0, (size_t)n_h, h_msm_out, false));
        zk_msm_last_stats(&ms_st);
        stats.msm_ms[3] = ms_st.total_device_ms;
    }
    worker.t.join();
    if (wit_rc != ZK_OK) {
        set_error("%s", wit_err.c_str());
        return wit_rc;
    }
    // device time of each witness MSM from the end of their shared sort (the
    // four run side by side, beside the work above)
    stats.msm_ms[0] = set_ms[0];
    stats.msm_ms[1] = set_ms[1];
    stats.msm_ms[4] = set_ms[2];
    stats.msm_ms[2] = set_ms[3];

    assemble(pk, r, s, a_msm, b_msm, l_msm, h_msm_out, b1_msm, outA, outB, outC);
    ZK_TRY_CUDA(cudaEventRecord(ev[3], st));
    if (st != user_st) ZK_TRY_CUDA(cudaStreamWaitEvent(user_st, ev[3], 0));
    ZK_TRY_CUDA(cudaEventSynchronize(ev[3]));
    // The first proof ran its H MSM without window tables: their build starts
    // now, on the key's own stream, and later proofs use them once it is done.
    // Started inside the proof, the build delayed it (a first allocation of
    // the witness context's scratch waits for the whole device).
    if (n_h > 0 && (size_t)n_h * 4 >= (size_t)pk->n_h * 3) {
        std::lock_guard<std::mutex> lock(pk->h_mu);
        ZK_TRY(start_h_tables_locked(pk, true));
    }
    cudaEventElapsedTime(&ms, ev[0], ev[3]);
    stats.total_ms = ms;
    return ZK_OK;
}

// 256-byte proof: A.x A.y B.x.c0 B.x.c1 B.y.c0 B.y.c1 C.x C.y, each 32 B
// standard form little-endian (groth16.cu:1058-1074)
static void serialize_proof(uint8_t* out, const uint64_t A[8], const uint64_t B[16], const uint64_t C[8]) {
    const uint64_t* src[8] = {A, A + 4, B, B + 4, B + 8, B + 12, C, C + 4};
    for (int k = 0; k < 8; k++) {
        zkh::Fe f;
        std::memcpy(f.v, src[k], 32);
        uint64_t s[4];
        zkh::to_std(zkh::kP, s, f);
        std::memcpy(out + 32 * k, s, 32);  // host is little-endian
    }
}

// ------------------------------------------------------------------ key files
// ZKMLPK3 (groth16.cu:1104-1180): magic "ZKMLPK3\0", u32 3, i32 n, i32 m,
// i32 num_public, G1 alpha beta delta, G2 beta gamma delta, vec G1 tau_g1,
// vec G2 tau_g2, vec G1 A, vec G1 B1, vec G2 B2, vec G1 L, vec G1 H; a G1 record
// is u8 infinity + x + y (standard form), G2 is u8 + x.c0 x.c1 y.c0 y.c1, a vec is
// i32 count + records.
static void put_fp_std(std::vector<uint8_t>& b, const uint64_t* mont) {
    zkh::Fe f;
    std::memcpy(f.v, mont, 32);
    uint64_t s[4];
    zkh::to_std(zkh::kP, s, f);
    const uint8_t* p = (const uint8_t*)s;
    b.insert(b.end(), p, p + 32);
}
static void put_g1(std::vector<uint8_t>& b, const uint64_t* rec) {
    bool inf = true;
    for (int i = 0; i < 8; i++) if (rec[i]) inf = false;
    b.push_back(inf ? 1 : 0);
    put_fp_std(b, rec);
    put_fp_std(b, rec + 4);
}
static void put_g2(std::vector<uint8_t>& b, const uint64_t* rec) {
    bool inf = true;
    for (int i = 0; i < 16; i++) if (rec[i]) inf = false;
    b.push_back(inf ? 1 : 0);
    for (int k = 0; k < 4; k++) put_fp_std(b, rec + 4 * k);
}
static void put_i32(std::vector<uint8_t>& b, int32_t v) {
    const uint8_t* p = (const uint8_t*)&v;
    b.insert(b.end(), p, p + 4);
}

static int pk_save(const zk_groth16_pk* pk, const char* path) {
    FILE* f = fopen(path, "wb");
    if (!f) { set_error("pk_save: cannot open %s", path); return ZK_ERR_INVALID; }
    std::vector<uint8_t> b;
    const char magic[8] = {'Z', 'K', 'M', 'L', 'P', 'K', '3', '\0'};
    b.insert(b.end(), magic, magic + 8);
    uint32_t version = 3;
    b.insert(b.end(), (uint8_t*)&version, (uint8_t*)&version + 4);
    put_i32(b, pk->num_constraints);
    put_i32(b, pk->m);
    put_i32(b, pk->num_public);
    put_g1(b, pk->alpha1);
    put_g1(b, pk->beta1);
    put_g1(b, pk->delta1);
    put_g2(b, pk->beta2);
    put_g2(b, pk->gamma2);
    put_g2(b, pk->delta2);
    put_i32(b, 0);  // tau_powers_g1: never kept (groth16.cu:510-513)
    put_i32(b, 2);  // tau_powers_g2 = [G2, tau G2] (groth16.cu:517-519)
    put_g2(b, pk->g2gen);
    put_g2(b, pk->tau2);
    bool ok = fwrite(b.data(), 1, b.size(), f) == b.size();
    auto dump_vec = [&](const uint8_t* dev, size_t count, bool g2) {
        std::vector<uint64_t> h(count * (g2 ? 16 : 8));
        if (count) cudaMemcpy(h.data(), dev, h.size() * 8, cudaMemcpyDeviceToHost);
        std::vector<uint8_t> o;
        o.reserve(4 + count * (g2 ? 129 : 65));
        put_i32(o, (int32_t)count);
        for (size_t i = 0; i < count; i++) {
            if (g2) put_g2(o, &h[i * 16]);
            else put_g1(o, &h[i * 8]);
        }
        ok = ok && fwrite(o.data(), 1, o.size(), f) == o.size();
    };
    const size_t m = (size_t)pk->m;
    dump_vec(pk->g1, m, false);                                   // A
    dump_vec(pk->g1 + m * 64, m, false);                          // B1
    dump_vec(pk->g2, m, true);                                    // B2
    dump_vec(pk->g1 + 2 * m * 64, (size_t)pk->l, false);          // L
    dump_vec(pk->g1 + (2 * m + pk->l) * 64, (size_t)pk->n_h, false);  // H
    fclose(f);
    if (!ok) { set_error("pk_save: write failed for %s", path); return ZK_ERR_INVALID; }
    return ZK_OK;
}

struct Reader {
    const uint8_t* p;
    size_t left;
    bool ok = true;
    void raw(void* dst, size_t n) {
        if (!ok || left < n) { ok = false; return; }
        std::memcpy(dst, p, n);
        p += n;
        left -= n;
    }
    int32_t i32() { int32_t v = 0; raw(&v, 4); return v; }
};

// parse into standard-form records (infinity -> all zero); Montgomery
// conversion happens on the device
static void get_g1(Reader& R, uint64_t* rec) {
    uint8_t inf = 0;
    R.raw(&inf, 1);
    R.raw(rec, 64);
    if (inf) std::memset(rec, 0, 64);
}
static void get_g2(Reader& R, uint64_t* rec) {
    uint8_t inf = 0;
    R.raw(&inf, 1);
    R.raw(rec, 128);
    if (inf) std::memset(rec, 0, 128);
}
static void std_to_mont_host(uint64_t* v, size_t fe_count) {
    for (size_t i = 0; i < fe_count; i++) {
        bool z = (v[4 * i] | v[4 * i + 1] | v[4 * i + 2] | v[4 * i + 3]) == 0;
        if (z) continue;
        zkh::Fe f;
        zkh::from_std(zkh::kP, f, v + 4 * i);
        std::memcpy(v + 4 * i, f.v, 32);
    }
}

// ZKMLPK3 records: u8 infinity flag + x (+ y) in standard form, 65 B (G1) or
// 129 B (G2).  One thread per record: the record's bytes from aligned 32-bit
// words (funnel shifts), then x R^2 R^-1 per coordinate (Montgomery form);
// a set flag gives the all-zero record.  raw must extend 8 bytes past the
// last record (the loader's staging slots do).
template <int kCoords>
__global__ void unpack_records_kernel(const uint8_t* __restrict__ raw, size_t count, uint64_t* __restrict__ out) {
    constexpr int kRec = 1 + 32 * kCoords;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
        const size_t start = i * kRec;
        const uint8_t flag = raw[start];
        // the coordinates' bytes from 4-byte aligned words (alignment of the
        // absolute address: a vector's records need not start on a word)
        const uintptr_t a = reinterpret_cast<uintptr_t>(raw + start + 1);
        const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
        const uint32_t sh = (uint32_t)(a & 3) * 8;
        Fp r2;
#pragma unroll
        for (int k = 0; k < 8; k++) r2.v[k] = ModP::r2(k);
#pragma unroll
        for (int c = 0; c < kCoords; c++) {
            Fp x;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const uint32_t lo = w[c * 8 + k], hi = w[c * 8 + k + 1];
                x.v[k] = sh ? __funnelshift_r(lo, hi, sh) : lo;
            }
            if (flag) {
                fset_zero(x);
            } else {
                fmul(x, x, r2);
            }
            fstore(reinterpret_cast<Fp*>(out) + i * kCoords + c, x);
        }
    }
}

static thread_local zk_pk_load_stats g_load_stats;

// Pinned host staging of the key loader: kBufs buffers, allocated by the first
// load of the process (or grown by a later one) and kept until exit, so that a
// load neither pins nor unpins host memory after the first.
struct PinnedStaging {
    static constexpr int kBufs = 3;
    std::mutex mu;
    uint8_t* p[kBufs] = {};
    size_t bytes = 0;
    int ensure(size_t need) {
        if (bytes >= need) return ZK_OK;
        for (auto& q : p) {
            if (q) cudaFreeHost(q);
            q = nullptr;
        }
        bytes = 0;
        for (auto& q : p) ZK_TRY_CUDA(cudaMallocHost(&q, need));
        bytes = need;
        return ZK_OK;
    }
};
static PinnedStaging& pinned_staging() {
    static PinnedStaging* s = new PinnedStaging();  // never destroyed: freed with the process
    return *s;
}

// ZKMLPK3 (ProvingKey::save / load_streaming, groth16.cu:1104-1314) straight
// into device memory: the header and vector counts are read first (fixed-size
// records give every offset), then the five query vectors in pieces of whole
// records (32 MiB at most): several threads read a piece into pinned staging,
// it is copied to a device staging slot, and a kernel unpacks its records
// into the key and converts them to Montgomery form, while the next piece is
// read.  Fail-closed as the reference's loader: bad magic or version, bad
// counts, truncation, incomplete query vectors.
static int pk_load(int device, const char* path, zk_groth16_pk* pk) {
    zk_pk_load_stats& st = g_load_stats;
    std::memset(&st, 0, sizeof st);
    const auto t0 = std::chrono::steady_clock::now();
    FILE* f = fopen(path, "rb");
    if (!f) { set_error("pk_load: cannot open %s", path); return ZK_ERR_INVALID; }
    struct Closer {
        FILE* f;
        ~Closer() { fclose(f); }
    } closer{f};
    fseek(f, 0, SEEK_END);
    const long long size = ftell(f);
    fseek(f, 0, SEEK_SET);
    auto rd = [&](void* p, size_t n) { return fread(p, 1, n, f) == n; };
    auto skip = [&](long long n) { return fseek(f, (long)n, SEEK_CUR) == 0; };
    auto rd_i32 = [&](int32_t& v) { return rd(&v, 4); };
    auto rd_rec = [&](uint64_t* rec, int coords) {
        uint8_t inf = 0;
        if (!rd(&inf, 1) || !rd(rec, (size_t)32 * coords)) return false;
        if (inf) std::memset(rec, 0, (size_t)32 * coords);
        return true;
    };
    char magic[8];
    uint32_t version = 0;
    if (!rd(magic, 8) || !rd(&version, 4) || std::memcmp(magic, "ZKMLPK3", 7) != 0 || version != 3) {
        set_error("pk_load: %s is not a ZKMLPK3 v3 proving key", path);
        return ZK_ERR_INVALID;
    }
    if (!rd_i32(pk->num_constraints) || !rd_i32(pk->m) || !rd_i32(pk->num_public) || pk->num_constraints < 0 || pk->m <= 0 ||
        pk->num_public < 0) {
        set_error("pk_load: invalid metadata in %s", path);
        return ZK_ERR_INVALID;
    }
    uint64_t small1[3][8], small2[3][16];
    bool ok = true;
    for (int k = 0; k < 3; k++) ok = ok && rd_rec(small1[k], 2);
    for (int k = 0; k < 3; k++) ok = ok && rd_rec(small2[k], 4);
    int32_t ntg1 = -1, ntg2 = -1;
    ok = ok && rd_i32(ntg1) && ntg1 >= 0 && ntg1 <= (1 << 28) && skip((long long)ntg1 * 65);
    if (!ok) { set_error("pk_load: bad header or tau_g1 vector in %s", path); return ZK_ERR_INVALID; }
    ok = rd_i32(ntg2) && ntg2 >= 0 && ntg2 <= (1 << 28);
    uint64_t tg2[2][16] = {};
    for (int32_t i = 0; ok && i < std::min(ntg2, 2); i++) ok = rd_rec(tg2[i], 4);
    ok = ok && (ntg2 <= 2 || skip((long long)(ntg2 - 2) * 129));
    if (!ok) { set_error("pk_load: bad tau_g2 vector in %s", path); return ZK_ERR_INVALID; }
    // the five query vectors: A, B1 (G1), B2 (G2), L, H (G1)
    int32_t counts[5];
    long long off[5];
    for (int v = 0; v < 5; v++) {
        const int rec = v == 2 ? 129 : 65;
        if (!rd_i32(counts[v]) || counts[v] < 0 || counts[v] > (1 << 28)) {
            set_error("pk_load: bad vector count in %s", path);
            return ZK_ERR_INVALID;
        }
        off[v] = ftell(f);
        if (off[v] + (long long)counts[v] * rec > size || !skip((long long)counts[v] * rec)) {
            set_error("pk_load: truncated file %s", path);
            return ZK_ERR_INVALID;
        }
    }
    if (counts[0] < pk->m || counts[1] < pk->m || counts[2] < pk->m) {
        set_error("pk_load: incomplete v3 proving key in %s", path);  // groth16.cu:1300-1305
        return ZK_ERR_INVALID;
    }
    if (counts[0] != pk->m || counts[1] != pk->m || counts[2] != pk->m) {
        set_error("pk_load: query vectors longer than num_variables are not supported");
        return ZK_ERR_RANGE;
    }
    pk->l = counts[3];
    pk->n_h = counts[4];
    std_to_mont_host(&small1[0][0], 6);
    std_to_mont_host(&small2[0][0], 12);
    std_to_mont_host(&tg2[0][0], 8);
    std::memcpy(pk->alpha1, small1[0], 64);
    std::memcpy(pk->beta1, small1[1], 64);
    std::memcpy(pk->delta1, small1[2], 64);
    std::memcpy(pk->beta2, small2[0], 128);
    std::memcpy(pk->gamma2, small2[1], 128);
    std::memcpy(pk->delta2, small2[2], 128);
    std::memcpy(pk->g2gen, tg2[0], 128);
    std::memcpy(pk->tau2, tg2[1], 128);

    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    pk->device = ctx->device;
    const size_t g1_count = (size_t)counts[0] + counts[1] + counts[3] + counts[4];
    DeviceBuffer g1_buf, g2_buf;
    const auto a0 = std::chrono::steady_clock::now();
    ZK_TRY_CUDA(g1_buf.alloc(std::max<size_t>(g1_count, 1) * 64));
    ZK_TRY_CUDA(g2_buf.alloc(std::max<size_t>(counts[2], 1) * 128));
    // ZKML_PK_LOAD_CHUNK_MB overrides the 32 MiB chunk
    const char* ce = getenv("ZKML_PK_LOAD_CHUNK_MB");
    const size_t chunk = (ce && atoi(ce) > 0 && atoi(ce) <= 4096 ? (size_t)atoi(ce) : (size_t)32) << 20;
    // a piece never exceeds the chunk nor the query vectors' total size
    const size_t total = ((size_t)counts[0] + counts[1] + counts[3] + counts[4]) * 65 + (size_t)counts[2] * 129;
    const size_t stage_bytes = std::max<size_t>(std::min(chunk, total), 1);
    PinnedStaging& pool = pinned_staging();
    std::lock_guard<std::mutex> pool_lock(pool.mu);
    ZK_TRY(pool.ensure(stage_bytes));
    const size_t slot = stage_bytes + 64;  // the unpack kernel reads up to 8 bytes past a piece's last record
    // the device slots live in the context's scratch arena (grown once, kept):
    // nothing is allocated or freed on the device for them after the first use
    std::lock_guard<std::mutex> ctx_lock(ctx->mu);
    ZK_TRY(ensure_scratch(ctx, PinnedStaging::kBufs * slot));
    cudaStream_t cs = ctx->copy_stream;
    ZK_TRY(scratch_begin(ctx, cs));
    uint8_t* stage = (uint8_t*)ctx->scratch;
    ZK_TRY_CUDA(cudaMemsetAsync(stage, 0, PinnedStaging::kBufs * slot, cs));
    cudaEvent_t slot_free[PinnedStaging::kBufs] = {};
    struct EventSet {
        cudaEvent_t* e;
        cudaStream_t s;
        ~EventSet() {
            cudaStreamSynchronize(s);  // no copy or kernel still uses the staging on any exit path
            for (int i = 0; i < PinnedStaging::kBufs; i++)
                if (e[i]) cudaEventDestroy(e[i]);
        }
    } events{slot_free, cs};
    for (int i = 0; i < PinnedStaging::kBufs; i++) {
        ZK_TRY_CUDA(cudaEventCreateWithFlags(&slot_free[i], cudaEventDisableTiming));
        ZK_TRY_CUDA(cudaEventRecord(slot_free[i], cs));
    }
    st.alloc_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - a0).count();
    // Pieces of whole records of one vector, at most a chunk each: kThreads
    // readers fill a pinned slot, the copy engine moves it to the device slot
    // and one kernel unpacks it into the key, while the next piece is read.
    // Output: A | B1 | L | H into g1 (file order A, B1, B2, L, H), B2 into g2.
    constexpr int kThreads = 8;
    const int fd = fileno(f);
    const int grid = ctx->num_sms * 8;
    const size_t g1_at[5] = {0, (size_t)counts[0], 0, (size_t)counts[0] + counts[1], (size_t)counts[0] + counts[1] + counts[3]};
    double read_s = 0, bytes = 0;
    size_t piece = 0;
    for (int v = 0; v < 5; v++) {
        const size_t rec = v == 2 ? 129 : 65;
        const size_t per = chunk / rec;
        for (size_t r0 = 0; r0 < (size_t)counts[v]; r0 += per, piece++) {
            const size_t nrec = std::min(per, (size_t)counts[v] - r0), len = nrec * rec;
            const long long at = off[v] + (long long)(r0 * rec);
            const int b = (int)(piece % PinnedStaging::kBufs);
            ZK_TRY_CUDA(cudaEventSynchronize(slot_free[b]));
            const auto r_start = std::chrono::steady_clock::now();
            std::atomic<bool> bad{false};
            {
                std::vector<std::thread> th;
                for (int t = 0; t < kThreads; t++)
                    th.emplace_back([&, t]() {
                        size_t x = len * t / kThreads, e = len * (t + 1) / kThreads;
                        while (x < e) {
                            const ssize_t got = pread(fd, pool.p[b] + x, e - x, (off_t)(at + (long long)x));
                            if (got <= 0) { bad = true; return; }
                            x += (size_t)got;
                        }
                    });
                for (auto& x : th) x.join();
            }
            read_s += std::chrono::duration<double>(std::chrono::steady_clock::now() - r_start).count();
            if (bad) { set_error("pk_load: read failed for %s", path); return ZK_ERR_INVALID; }
            bytes += (double)len;
            uint8_t* dslot = stage + (size_t)b * slot;
            ZK_TRY_CUDA(cudaMemcpyAsync(dslot, pool.p[b], len, cudaMemcpyHostToDevice, cs));
            if (v == 2)
                unpack_records_kernel<4><<<grid, 256, 0, cs>>>(dslot, nrec, (uint64_t*)((uint8_t*)g2_buf.p + r0 * 128));
            else
                unpack_records_kernel<2><<<grid, 256, 0, cs>>>(dslot, nrec, (uint64_t*)((uint8_t*)g1_buf.p + (g1_at[v] + r0) * 64));
            ZK_TRY_CUDA(cudaGetLastError());
            ZK_TRY_CUDA(cudaEventRecord(slot_free[b], cs));
        }
    }
    ZK_TRY(scratch_end(ctx, cs));
    ZK_TRY_CUDA(cudaStreamSynchronize(cs));
    pk->g1 = (uint8_t*)g1_buf.release();
    pk->g2 = (uint8_t*)g2_buf.release();
    st.bytes = bytes;
    st.read_ms = read_s * 1e3;
    st.total_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return ZK_OK;
}

// vk.bin (src/verifier/verifier.cu:103-148): i32 num_public, alpha1 (x, y),
// beta2 gamma2 delta2 (x.c0 x.c1 y.c0 y.c1), i32 num_ic, ic[] (x, y); standard
// form, no infinity flags
static int vk_save(const zk_groth16_pk* pk, const char* path) {
    if (pk->ic.empty()) { set_error("vk_save: this proving key carries no verification key (loaded from a file)"); return ZK_ERR_INVALID; }
    std::vector<uint8_t> b;
    put_i32(b, pk->num_public);
    put_fp_std(b, pk->alpha1);
    put_fp_std(b, pk->alpha1 + 4);
    for (const uint64_t* g : {pk->beta2, pk->gamma2, pk->delta2})
        for (int k = 0; k < 4; k++) put_fp_std(b, g + 4 * k);
    const int nic = (int)(pk->ic.size() / 8);
    put_i32(b, nic);
    for (int i = 0; i < nic; i++) {
        put_fp_std(b, &pk->ic[(size_t)i * 8]);
        put_fp_std(b, &pk->ic[(size_t)i * 8 + 4]);
    }
    FILE* f = fopen(path, "wb");
    if (!f) { set_error("vk_save: cannot open %s", path); return ZK_ERR_INVALID; }
    const bool ok = fwrite(b.data(), 1, b.size(), f) == b.size();
    fclose(f);
    return ok ? ZK_OK : ZK_ERR_INVALID;
}

}  // namespace zk

// ================================================================== C ABI
using namespace zk;

extern "C" int zk_r1cs_create(int device, int num_constraints, int num_variables, int num_public, const void* a_entries,
                              size_t a_nnz, const void* b_entries, size_t b_nnz, const void* c_entries, size_t c_nnz,
                              zk_r1cs** out) {
    clear_error();
    if (!out || (a_nnz && !a_entries) || (b_nnz && !b_entries) || (c_nnz && !c_entries)) return ZK_ERR_INVALID;
    zk_r1cs* r = new zk_r1cs();
    const SparseEntry* ent[3] = {(const SparseEntry*)a_entries, (const SparseEntry*)b_entries, (const SparseEntry*)c_entries};
    const size_t nnz[3] = {a_nnz, b_nnz, c_nnz};
    int st = r1cs_create(device, num_constraints, num_variables, num_public, ent, nnz, r->r);
    if (st != ZK_OK) { zk_r1cs_destroy(r); return st; }
    *out = r;
    return ZK_OK;
}

extern "C" void zk_r1cs_destroy(zk_r1cs* r) {
    if (!r) return;
    for (int k = 0; k < 3; k++) {
        cudaFree(r->r.d_row_ptr[k]);
        cudaFree(r->r.d_col[k]);
        cudaFree(r->r.d_val[k]);
        cudaFree(r->r.d_mid[k]);
        cudaFree(r->r.d_long[k]);
    }
    delete r;
}

extern "C" int zk_r1cs_domain(const zk_r1cs* r, int* log_n) {
    if (!r || !log_n) return ZK_ERR_INVALID;
    *log_n = r->r.log_n;
    return ZK_OK;
}

extern "C" int zk_groth16_setup(zk_r1cs* r1cs, const void* toxic, zk_groth16_pk** out) {
    clear_error();
    if (!r1cs || !toxic || !out) return ZK_ERR_INVALID;
    zkh::Fe tx[5];
    std::memcpy(tx, toxic, sizeof tx);
    zk_groth16_pk* pk = new zk_groth16_pk();
    int st = setup(r1cs->r, tx, pk);
    if (st != ZK_OK) { zk_groth16_pk_destroy(pk); return st; }
    *out = pk;
    return ZK_OK;
}

extern "C" int zk_groth16_pk_load(int device, const char* path, zk_groth16_pk** out) {
    clear_error();
    if (!path || !out) return ZK_ERR_INVALID;
    zk_groth16_pk* pk = new zk_groth16_pk();
    int st = pk_load(device, path, pk);
    if (st != ZK_OK) { zk_groth16_pk_destroy(pk); return st; }
    *out = pk;
    return ZK_OK;
}

extern "C" int zk_groth16_pk_last_load_stats(zk_pk_load_stats* out) {
    if (!out) return ZK_ERR_INVALID;
    *out = g_load_stats;
    return ZK_OK;
}

extern "C" int zk_groth16_pk_save(const zk_groth16_pk* pk, const char* path) {
    clear_error();
    if (!pk || !path) return ZK_ERR_INVALID;
    DeviceContext* ctx;
    ZK_TRY(get_context(pk->device, &ctx));
    return pk_save(pk, path);
}

extern "C" int zk_groth16_vk_save(const zk_groth16_pk* pk, const char* path) {
    clear_error();
    if (!pk || !path) return ZK_ERR_INVALID;
    return vk_save(pk, path);
}

extern "C" int zk_groth16_vk_points(const zk_groth16_pk* pk, void* alpha1, void* beta2, void* gamma2, void* delta2, void* ic,
                                    int ic_capacity) {
    if (!pk) return ZK_ERR_INVALID;
    if (alpha1) std::memcpy(alpha1, pk->alpha1, 64);
    if (beta2) std::memcpy(beta2, pk->beta2, 128);
    if (gamma2) std::memcpy(gamma2, pk->gamma2, 128);
    if (delta2) std::memcpy(delta2, pk->delta2, 128);
    const int nic = (int)(pk->ic.size() / 8);
    if (ic) std::memcpy(ic, pk->ic.data(), (size_t)std::min(nic, std::max(ic_capacity, 0)) * 64);
    return nic;
}

extern "C" void zk_groth16_pk_destroy(zk_groth16_pk* pk) {
    if (!pk) return;
    if (pk->device >= 0) cudaSetDevice(pk->device);
    cudaFree(pk->g1);
    cudaFree(pk->g2);
    cudaFree(pk->w);
    cudaFree(pk->abc);
    cudaFree(pk->h);
    cudaFree(pk->d_bad);
    cudaFreeHost(pk->h_bad);
    if (pk->h_tab_stream) cudaStreamSynchronize(pk->h_tab_stream);
    if (pk->prio_stream) {
        cudaStreamSynchronize(pk->prio_stream);
        cudaStreamDestroy(pk->prio_stream);
    }
    cudaFree(pk->h_tab);
    cudaFree(pk->h_tab_pending);
    if (pk->h_tab_done) cudaEventDestroy(pk->h_tab_done);
    if (pk->h_tab_stream) cudaStreamDestroy(pk->h_tab_stream);
    for (auto& kv : pk->hb) {
        cudaFree(kv.second.pts);
        cudaFree(kv.second.tab);
    }
    zk::destroy_split_states(pk);
    zk::destroy_context(pk->wctx);
    delete pk;
}

extern "C" int zk_groth16_prove(zk_groth16_pk* pk, const zk_r1cs* r1cs, void* stream, const void* h_witness, const void* r,
                                const void* s, void* proof256, void* points) {
    clear_error();
    if (!pk || !r1cs || !h_witness || !r || !s || !proof256) return ZK_ERR_INVALID;
    zkh::Fe rr, ss;
    std::memcpy(rr.v, r, 32);
    std::memcpy(ss.v, s, 32);
    uint64_t A[8], B[16], C[8];
    ZK_TRY(prove(pk, r1cs->r, (cudaStream_t)stream, h_witness, rr, ss, A, B, C));
    serialize_proof((uint8_t*)proof256, A, B, C);
    if (points) {
        uint64_t* p = (uint64_t*)points;
        std::memcpy(p, A, 64);
        std::memcpy(p + 8, B, 128);
        std::memcpy(p + 24, C, 64);
    }
    return ZK_OK;
}

extern "C" int zk_groth16_last_stats(zk_prove_stats* out) {
    if (!out) return ZK_ERR_INVALID;
    *out = g_prove_stats;
    return ZK_OK;
}

// ------------------------------------------------------------------ pieces of a prove split across devices
extern "C" int zk_r1cs_matvec_rows_device(const zk_r1cs* r1cs, void* stream, const void* d_witness, uint64_t row_lo, uint64_t row_hi,
                                          void* d_out3) {
    clear_error();
    if (!r1cs || !d_witness || (!d_out3 && row_hi > row_lo)) return ZK_ERR_INVALID;
    const R1cs& R = r1cs->r;
    if (row_lo > row_hi || row_hi > R.n) {
        set_error("matvec: rows [%llu, %llu) outside the domain of %llu", (unsigned long long)row_lo, (unsigned long long)row_hi,
                  (unsigned long long)R.n);
        return ZK_ERR_RANGE;
    }
    DeviceContext* ctx;
    ZK_TRY(get_context(R.device, &ctx));
    return r1cs_matvec_rows(R, (cudaStream_t)stream, (const Fr*)d_witness, row_lo, row_hi, (Fr*)d_out3, ctx->num_sms);
}

extern "C" int zk_fr_hadamard_check_device(int device, void* stream, const void* d_a, const void* d_b, const void* d_c, size_t count,
                                           uint64_t row0, long long* first_bad) {
    clear_error();
    if (!first_bad || (count && (!d_a || !d_b || !d_c))) return ZK_ERR_INVALID;
    *first_bad = -1;
    if (!count) return ZK_OK;
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    cudaStream_t st = (cudaStream_t)stream;
    PoolBuffer bad_buf;
    ZK_TRY_CUDA(bad_buf.alloc(sizeof(unsigned long long), st));
    unsigned long long* d_bad = (unsigned long long*)bad_buf.p;
    ZK_TRY_CUDA(cudaMemsetAsync(d_bad, 0xff, sizeof(unsigned long long), st));
    enqueue_hadamard_check(st, (const Fr*)d_a, (const Fr*)d_b, (const Fr*)d_c, count, row0, d_bad, ctx->num_sms);
    unsigned long long bad = 0;
    ZK_TRY_CUDA(cudaMemcpyAsync(&bad, d_bad, sizeof bad, cudaMemcpyDeviceToHost, st));
    ZK_TRY_CUDA(cudaStreamSynchronize(st));
    *first_bad = bad == ~0ull ? -1 : (long long)bad;
    return ZK_OK;
}

extern "C" int zk_groth16_pk_arrays(const zk_groth16_pk* pk, zk_groth16_arrays* out) {
    clear_error();
    if (!pk || !out) return ZK_ERR_INVALID;
    out->device = pk->device;
    out->m = pk->m;
    out->num_public = pk->num_public;
    out->l = pk->l;
    out->n_h = pk->n_h;
    out->a = pk->g1;
    out->b1 = pk->g1 + (size_t)pk->m * 64;
    out->l_query = pk->g1 + 2 * (size_t)pk->m * 64;
    out->h_query = pk->g1 + (2 * (size_t)pk->m + pk->l) * 64;
    out->b2 = pk->g2;
    return ZK_OK;
}

extern "C" int zk_groth16_assemble_parts(const zk_groth16_pk* pk, const void* r, const void* s, const void* parts, int nparts,
                                         void* proof256, void* points) {
    clear_error();
    if (!pk || !r || !s || !proof256 || nparts < 0 || (nparts && !parts)) return ZK_ERR_INVALID;
    zkh::Fe rr, ss;
    std::memcpy(rr.v, r, 32);
    std::memcpy(ss.v, s, 32);
    zkh::Xyzz<zkh::Fe> a, l, h, b1, t;
    zkh::Xyzz<zkh::Fp2> b, t2;
    zkh::set_identity(a);
    zkh::set_identity(l);
    zkh::set_identity(h);
    zkh::set_identity(b1);
    zkh::set_identity(b);
    for (int i = 0; i < nparts; i++) {  // A (8) | B2 (16) | L (8) | H (8) | B1 (8) words per part
        const uint64_t* q = (const uint64_t*)parts + (size_t)i * 48;
        load_aff(t, q);
        zkh::add(a, t);
        load_aff(t2, q + 8);
        zkh::add(b, t2);
        load_aff(t, q + 24);
        zkh::add(l, t);
        load_aff(t, q + 32);
        zkh::add(h, t);
        load_aff(t, q + 40);
        zkh::add(b1, t);
    }
    uint64_t A[8], B[16], C[8];
    assemble_xyzz(pk, rr, ss, a, b, l, h, b1, A, B, C);
    serialize_proof((uint8_t*)proof256, A, B, C);
    if (points) {
        uint64_t* p = (uint64_t*)points;
        std::memcpy(p, A, 64);
        std::memcpy(p + 8, B, 128);
        std::memcpy(p + 24, C, 64);
    }
    return ZK_OK;
}

extern "C" int zk_groth16_assemble(const zk_groth16_pk* pk, const void* r, const void* s, const void* sums, void* proof256,
                                   void* points) {
    clear_error();
    if (!pk || !r || !s || !sums || !proof256) return ZK_ERR_INVALID;
    zkh::Fe rr, ss;
    std::memcpy(rr.v, r, 32);
    std::memcpy(ss.v, s, 32);
    const uint64_t* q = (const uint64_t*)sums;  // A (8) | B2 (16) | L (8) | H (8) | B1 (8) words
    uint64_t A[8], B[16], C[8];
    assemble(pk, rr, ss, q, q + 8, q + 24, q + 32, q + 40, A, B, C);
    serialize_proof((uint8_t*)proof256, A, B, C);
    if (points) {
        uint64_t* p = (uint64_t*)points;
        std::memcpy(p, A, 64);
        std::memcpy(p + 8, B, 128);
        std::memcpy(p + 24, C, 64);
    }
    return ZK_OK;
}

extern "C" int zk_groth16_precompute(zk_groth16_pk* pk, void* stream) {
    clear_error();
    if (!pk) return ZK_ERR_INVALID;
    DeviceContext* ctx;
    ZK_TRY(get_context(pk->device, &ctx));
    (void)stream;  // the tables are built on the key's own stream; this call returns when they are ready
    return ensure_h_tables(pk);
}

extern "C" int zk_groth16_h_msm_device(zk_groth16_pk* pk, void* stream, const void* d_h, uint64_t lo, uint64_t hi, void* out_affine) {
    clear_error();
    if (!pk || !out_affine || (hi > lo && !d_h)) return ZK_ERR_INVALID;
    if (lo > hi || hi > (uint64_t)pk->n_h) {
        set_error("h_msm: [%llu, %llu) outside the %d-point H query", (unsigned long long)lo, (unsigned long long)hi, pk->n_h);
        return ZK_ERR_RANGE;
    }
    DeviceContext* ctx;
    ZK_TRY(get_context(pk->device, &ctx));
    return h_msm(pk, (cudaStream_t)stream, (const Fr*)d_h, lo, hi, (uint64_t*)out_affine, true);
}

extern "C" int zk_groth16_h_msm_blocks_device(zk_groth16_pk* pk, void* stream, const void* d_h_part, int log_parts, int part,
                                              void* out_affine) {
    clear_error();
    if (!pk || !d_h_part || !out_affine) return ZK_ERR_INVALID;
    DeviceContext* ctx;
    ZK_TRY(get_context(pk->device, &ctx));
    return h_msm_blocks(pk, (cudaStream_t)stream, (const Fr*)d_h_part, log_parts, part, (uint64_t*)out_affine);
}

extern "C" int zk_groth16_witness_msms_device(zk_groth16_pk* pk, void* stream, const void* d_witness, uint64_t lo, uint64_t hi,
                                              void* sums) {
    clear_error();
    if (!pk || !sums || (hi > lo && !d_witness)) return ZK_ERR_INVALID;
    DeviceContext* ctx;
    ZK_TRY(get_context(pk->device, &ctx));
    ZK_TRY(ensure_witness_context(pk));
    uint64_t* q = (uint64_t*)sums;  // A (8) | B2 (16) | L (8) | H (8, untouched) | B1 (8) words
    float set_ms[4], all = 0;
    return witness_msms(pk, pk->wctx, (cudaStream_t)stream, (const Fr*)d_witness, lo, hi, q, q + 8, q + 40, q + 24, set_ms,
                        &all);
}
