// runtime.cu -- device contexts, scratch arenas, error channel, and the small
// C-ABI utilities (version, device count, last error, IMAD-rate probe).
#include "field.cuh"
#include "runtime.cuh"

#include <cstring>
#include <string>
#include <vector>

namespace zk {

static thread_local char g_err[512];
static thread_local MsmStats g_msm_stats;

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}
void clear_error() { g_err[0] = 0; }
MsmStats& msm_stats() { return g_msm_stats; }

static std::mutex g_ctx_mu;
static DeviceContext* g_ctx[64];

// Streams, events and device properties of a new context on `device`.
static int init_context(DeviceContext* c, int device) {
    c->device = device;
    cudaDeviceProp prop;
    ZK_TRY_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10) {
        set_error("device %d is sm_%d%d; this library is built for sm_100a only", device, prop.major, prop.minor);
        return ZK_ERR_NODEV;
    }
    c->num_sms = prop.multiProcessorCount;
    // keep stream-ordered allocations cached in the device's default pool
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
        uint64_t keep = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    ZK_TRY_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    ZK_TRY_CUDA(cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking));
    ZK_TRY_CUDA(cudaEventCreateWithFlags(&c->ev_a, cudaEventDisableTiming));
    ZK_TRY_CUDA(cudaEventCreateWithFlags(&c->ev_b, cudaEventDisableTiming));
    ZK_TRY_CUDA(cudaEventCreateWithFlags(&c->ev_c, cudaEventDisableTiming));
    ZK_TRY_CUDA(cudaEventCreateWithFlags(&c->scratch_done, cudaEventDisableTiming));
    ZK_TRY_CUDA(cudaEventRecord(c->scratch_done, c->stream));
    for (int i = 0; i < 9; i++) ZK_TRY_CUDA(cudaEventCreate(&c->phase[i]));
    ZK_TRY_CUDA(cudaStreamCreateWithFlags(&c->aux_stream, cudaStreamNonBlocking));
    for (int i = 0; i < 12; i++) ZK_TRY_CUDA(cudaEventCreateWithFlags(&c->batch_ev[i], cudaEventDisableTiming));
    return ZK_OK;
}

static int check_device(int& device) {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        set_error("no usable CUDA device (%s)", e == cudaSuccess ? "device count is 0" : cudaGetErrorString(e));
        return ZK_ERR_NODEV;
    }
    if (device < 0) ZK_TRY_CUDA(cudaGetDevice(&device));
    if (device >= count || device >= 64) {
        set_error("device %d out of range (%d visible)", device, count);
        return ZK_ERR_INVALID;
    }
    ZK_TRY_CUDA(cudaSetDevice(device));
    return ZK_OK;
}

int get_context(int device, DeviceContext** out) {
    ZK_TRY(check_device(device));
    std::lock_guard<std::mutex> lock(g_ctx_mu);
    if (!g_ctx[device]) {
        DeviceContext* c = new DeviceContext();
        const int rc = init_context(c, device);
        if (rc != ZK_OK) {
            destroy_context(c);
            return rc;
        }
        g_ctx[device] = c;
    }
    *out = g_ctx[device];
    return ZK_OK;
}

int create_context(int device, DeviceContext** out) {
    ZK_TRY(check_device(device));
    DeviceContext* c = new DeviceContext();
    const int rc = init_context(c, device);
    if (rc != ZK_OK) {
        destroy_context(c);
        return rc;
    }
    *out = c;
    return ZK_OK;
}

int ensure_set_streams(DeviceContext* ctx) {
    for (auto& s : ctx->set_stream)
        if (!s) ZK_TRY_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    return ZK_OK;
}

void destroy_context(DeviceContext* c) {
    if (!c) return;
    if (c->device >= 0) cudaSetDevice(c->device);
    for (cudaStream_t s : c->set_stream)
        if (s) {
            cudaStreamSynchronize(s);
            cudaStreamDestroy(s);
        }
    cudaStream_t streams[3] = {c->stream, c->copy_stream, c->aux_stream};
    for (cudaStream_t s : streams)
        if (s) cudaStreamSynchronize(s);
    release_ntt_tables(c);
    if (c->scratch) cudaFree(c->scratch);
    if (c->pinned) cudaFreeHost(c->pinned);
    cudaEvent_t evs[4] = {c->ev_a, c->ev_b, c->ev_c, c->scratch_done};
    for (cudaEvent_t e : evs)
        if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : c->phase)
        if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : c->batch_ev)
        if (e) cudaEventDestroy(e);
    for (cudaStream_t s : streams)
        if (s) cudaStreamDestroy(s);
    delete c;
}

int ensure_scratch(DeviceContext* ctx, size_t bytes) {
    if (ctx->scratch_bytes >= bytes) return ZK_OK;
    ZK_TRY_CUDA(cudaDeviceSynchronize());
    if (ctx->scratch) ZK_TRY_CUDA(cudaFree(ctx->scratch));
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
    size_t want = bytes + bytes / 8;  // headroom against small growth
    cudaError_t e = cudaMalloc(&ctx->scratch, want);
    if (e != cudaSuccess) {
        cudaGetLastError();
        e = cudaMalloc(&ctx->scratch, bytes);
        want = bytes;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        ctx->scratch = nullptr;
        set_error("scratch allocation of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
        return ZK_ERR_NOMEM;
    }
    ctx->scratch_bytes = want;
    return ZK_OK;
}

int scratch_begin(DeviceContext* ctx, cudaStream_t st) {
    ZK_TRY_CUDA(cudaStreamWaitEvent(st, ctx->scratch_done, 0));
    return ZK_OK;
}
int scratch_end(DeviceContext* ctx, cudaStream_t st) {
    ZK_TRY_CUDA(cudaEventRecord(ctx->scratch_done, st));
    return ZK_OK;
}

int ensure_pinned(DeviceContext* ctx, size_t bytes) {
    if (ctx->pinned_bytes >= bytes) return ZK_OK;
    if (ctx->pinned) cudaFreeHost(ctx->pinned);
    ctx->pinned = nullptr;
    ctx->pinned_bytes = 0;
    cudaError_t e = cudaMallocHost(&ctx->pinned, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("pinned staging allocation of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
        return ZK_ERR_NOMEM;
    }
    ctx->pinned_bytes = bytes;
    return ZK_OK;
}

// ------------------------------------------------------------------ IMAD probe
// The probe times the Montgomery multiplication of field.cuh itself (the inlined
// body; 8 rows of 2 x 16 IMAD) on 4 independent chains x <- x * y per thread at
// full occupancy, and reports 256 IMAD per multiplication.  This mix of paired
// mad.lo.cc / madc.hi.cc chains sustains more than plain mad.hi (half rate on
// B200) and is the honest ceiling for every kernel built on it.
__global__ void __launch_bounds__(256) imad_probe_kernel(uint32_t* out, uint32_t seed, int iters) {
    Fp x[4], y;
#pragma unroll
    for (int k = 0; k < 8; k++) y.v[k] = (seed * (k + 3) + threadIdx.x) & 0x0fffffffu;
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
        for (int k = 0; k < 8; k++) x[j].v[k] = (seed + j * 9 + k + blockIdx.x) & 0x0fffffffu;
    for (int i = 0; i < iters; i++) {
#pragma unroll
        for (int j = 0; j < 4; j++) fmul_inline(x[j], x[j], y);
    }
    uint32_t acc = 0;
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
        for (int k = 0; k < 8; k++) acc ^= x[j].v[k];
    out[blockIdx.x * blockDim.x + threadIdx.x] = acc;
}

// ------------------------------------------------------------------ INT32 pipe probe
// The hardware issue rate of the 32-bit integer multiply-add, independent of
// any field code: 8 independent chains per thread at full occupancy, each step
// one instruction of the probed form (kMode 0: mad.lo.u32; 1: mad.hi.u32;
// 2: a mad.lo.cc.u32 / madc.hi.u32 pair, the two halves of one 32 x 32-bit
// product with carry, counted as 2 instructions).  Thread 0 of each block
// records clock64 and the global timer around its loop, giving the SM clock
// the probe ran at.
template <int kMode>
__global__ void __launch_bounds__(256) int_pipe_probe_kernel(uint32_t* out, unsigned long long* clk, uint32_t seed, int iters) {
    uint32_t a[8];
    const uint32_t m = seed | 1u;
#pragma unroll
    for (int k = 0; k < 8; k++) a[k] = seed * (k + 1) + threadIdx.x + blockIdx.x;
    unsigned long long c0 = 0, t0 = 0;
    if (threadIdx.x == 0) {
        c0 = clock64();
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    }
    for (int i = 0; i < iters; i++) {
#pragma unroll
        for (int r = 0; r < 4; r++) {
#pragma unroll
            for (int k = 0; k < 8; k++) {
                if (kMode == 0) {
                    asm volatile("mad.lo.u32 %0, %0, %1, %2;" : "+r"(a[k]) : "r"(m), "r"((uint32_t)k));
                } else if (kMode == 1) {
                    asm volatile("mad.hi.u32 %0, %0, %1, %2;" : "+r"(a[k]) : "r"(m), "r"((uint32_t)k));
                } else {
                    asm volatile("{\n\t.reg .u32 t;\n\t"
                                 "mad.lo.cc.u32 t, %0, %1, %2;\n\t"
                                 "madc.hi.u32 %0, %0, %1, t;\n\t}"
                                 : "+r"(a[k]) : "r"(m), "r"((uint32_t)k));
                }
            }
        }
    }
    if (threadIdx.x == 0) {
        unsigned long long c1 = clock64(), t1;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
        clk[2 * blockIdx.x] = c1 - c0;
        clk[2 * blockIdx.x + 1] = t1 - t0;
    }
    uint32_t acc = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) acc ^= a[k];
    out[blockIdx.x * blockDim.x + threadIdx.x] = acc;
}

template <int kMode>
static int run_int_pipe_probe(DeviceContext* ctx, uint32_t* buf, unsigned long long* clk_dev, double* per_s, double* ghz) {
    const int threads = 256, blocks = ctx->num_sms * 8, iters = 512;
    ScopedEvent a, b;
    ZK_TRY_CUDA(cudaEventCreate(&a.e));
    ZK_TRY_CUDA(cudaEventCreate(&b.e));
    int_pipe_probe_kernel<kMode><<<blocks, threads, 0, ctx->stream>>>(buf, clk_dev, 12345u, 64);  // warm-up
    ZK_TRY_CUDA(cudaEventRecord(a.e, ctx->stream));
    int_pipe_probe_kernel<kMode><<<blocks, threads, 0, ctx->stream>>>(buf, clk_dev, 777u, iters);
    ZK_TRY_CUDA(cudaEventRecord(b.e, ctx->stream));
    ZK_TRY_CUDA(cudaEventSynchronize(b.e));
    float ms = 0;
    cudaEventElapsedTime(&ms, a.e, b.e);
    const double per_step = kMode == 2 ? 2.0 : 1.0;
    *per_s = (double)threads * blocks * iters * 4 * 8 * per_step / (ms * 1e-3);
    std::vector<unsigned long long> clk((size_t)2 * blocks);
    ZK_TRY_CUDA(cudaMemcpy(clk.data(), clk_dev, clk.size() * 8, cudaMemcpyDeviceToHost));
    double cyc = 0, ns = 0;
    for (int i = 0; i < blocks; i++) {
        cyc += (double)clk[(size_t)2 * i];
        ns += (double)clk[(size_t)2 * i + 1];
    }
    *ghz = ns > 0 ? cyc / ns : 0.0;
    return ZK_OK;
}

}  // namespace zk

using namespace zk;

extern "C" int zk_probe_int_pipe(int device, zk_int_pipe_rates* out) {
    clear_error();
    if (!out) return ZK_ERR_INVALID;
    std::memset(out, 0, sizeof *out);
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    std::lock_guard<std::mutex> lock(ctx->mu);
    const int blocks = ctx->num_sms * 8;
    PoolBuffer ob, cb;
    ZK_TRY_CUDA(ob.alloc((size_t)256 * blocks * 4, ctx->stream));
    ZK_TRY_CUDA(cb.alloc((size_t)2 * blocks * 8, ctx->stream));
    double ghz[3] = {0, 0, 0};
    ZK_TRY(run_int_pipe_probe<0>(ctx, (uint32_t*)ob.p, (unsigned long long*)cb.p, &out->mad_lo_per_s, &ghz[0]));
    ZK_TRY(run_int_pipe_probe<1>(ctx, (uint32_t*)ob.p, (unsigned long long*)cb.p, &out->mad_hi_per_s, &ghz[1]));
    ZK_TRY(run_int_pipe_probe<2>(ctx, (uint32_t*)ob.p, (unsigned long long*)cb.p, &out->mad_pair_per_s, &ghz[2]));
    out->num_sms = ctx->num_sms;
    out->sm_clock_ghz = (ghz[0] + ghz[1] + ghz[2]) / 3.0;
    const double per_clk = (double)ctx->num_sms * out->sm_clock_ghz * 1e9;
    if (per_clk > 0) {
        out->mad_lo_per_clk_sm = out->mad_lo_per_s / per_clk;
        out->mad_hi_per_clk_sm = out->mad_hi_per_s / per_clk;
        out->mad_pair_per_clk_sm = out->mad_pair_per_s / per_clk;
    }
    return ZK_OK;
}

extern "C" const char* zk_last_error(void) { return g_err; }

extern "C" int zk_version(void) { return 100; }

extern "C" int zk_device_count(int* count) {
    clear_error();
    if (!count) return ZK_ERR_INVALID;
    int c = 0;
    cudaError_t e = cudaGetDeviceCount(&c);
    if (e != cudaSuccess) {
        cudaGetLastError();
        c = 0;
    }
    *count = c;
    return ZK_OK;
}

extern "C" int zk_probe_imad_rate(int device, double* rate) {
    clear_error();
    if (!rate) return ZK_ERR_INVALID;
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    std::lock_guard<std::mutex> lock(ctx->mu);
    const int threads = 256, blocks = ctx->num_sms * 8, iters = 256;
    PoolBuffer out;
    ZK_TRY_CUDA(out.alloc((size_t)threads * blocks * 4, ctx->stream));
    uint32_t* buf = (uint32_t*)out.p;
    ScopedEvent a, b;
    ZK_TRY_CUDA(cudaEventCreate(&a.e));
    ZK_TRY_CUDA(cudaEventCreate(&b.e));
    imad_probe_kernel<<<blocks, threads, 0, ctx->stream>>>(buf, 12345u, 64);  // warm-up
    ZK_TRY_CUDA(cudaEventRecord(a.e, ctx->stream));
    imad_probe_kernel<<<blocks, threads, 0, ctx->stream>>>(buf, 777u, iters);
    ZK_TRY_CUDA(cudaEventRecord(b.e, ctx->stream));
    ZK_TRY_CUDA(cudaEventSynchronize(b.e));
    float ms = 0;
    cudaEventElapsedTime(&ms, a.e, b.e);
    double instr = (double)threads * blocks * iters * 4 * 256.0;  // 4 chains x 256 IMAD per multiplication
    *rate = instr / (ms * 1e-3);
    return ZK_OK;
}
