// runtime.cu -- device contexts, scratch arenas, error channel, and the small
// C-ABI utilities (version, device count, last error, IMAD-rate probe).
#include "field.cuh"
#include "runtime.cuh"

#include <cstring>
#include <string>

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

void destroy_context(DeviceContext* c) {
    if (!c) return;
    if (c->device >= 0) cudaSetDevice(c->device);
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

}  // namespace zk

using namespace zk;

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
