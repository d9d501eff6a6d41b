// runtime.cuh -- per-device context of the B200 prover runtime: streams, a
// growable device scratch arena, pinned host staging, cached NTT tables and
// the thread-local error channel behind the C ABI's status codes.
#pragma once
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../include/zkml_b200.h"

namespace zk {

void set_error(const char* fmt, ...);
void clear_error();

#define ZK_TRY_CUDA(call)                                                                \
    do {                                                                                 \
        cudaError_t e_ = (call);                                                         \
        if (e_ != cudaSuccess) {                                                         \
            ::zk::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call, cudaGetErrorString(e_)); \
            return e_ == cudaErrorMemoryAllocation ? ZK_ERR_NOMEM : ZK_ERR_CUDA;         \
        }                                                                                \
    } while (0)

#define ZK_TRY(call)                 \
    do {                             \
        int s_ = (call);             \
        if (s_ != ZK_OK) return s_;  \
    } while (0)

// A CUDA event owned by a scope: destroyed on every exit path, errors included.
struct ScopedEvent {
    cudaEvent_t e = nullptr;
    ScopedEvent() = default;
    ScopedEvent(const ScopedEvent&) = delete;
    ScopedEvent& operator=(const ScopedEvent&) = delete;
    ~ScopedEvent() {
        if (e) cudaEventDestroy(e);
    }
};

// A stream-ordered pool allocation owned by a scope: returned with
// cudaFreeAsync on its stream (after the work queued there) on every exit path.
struct PoolBuffer {
    void* p = nullptr;
    cudaStream_t st = nullptr;
    PoolBuffer() = default;
    PoolBuffer(const PoolBuffer&) = delete;
    PoolBuffer& operator=(const PoolBuffer&) = delete;
    ~PoolBuffer() {
        if (p) cudaFreeAsync(p, st);
    }
    cudaError_t alloc(size_t bytes, cudaStream_t stream) {
        st = stream;
        return cudaMallocAsync(&p, bytes, stream);
    }
};

// A cudaMalloc allocation owned by a scope: freed on every exit path unless
// release() hands it on.
struct DeviceBuffer {
    void* p = nullptr;
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer() {
        if (p) cudaFree(p);
    }
    cudaError_t alloc(size_t bytes) { return cudaMalloc(&p, bytes); }
    void* release() {
        void* q = p;
        p = nullptr;
        return q;
    }
};

// bump allocator over one device buffer; all offsets 256-byte aligned
struct Arena {
    char* base = nullptr;
    size_t used = 0;
    template <class T>
    T* take(size_t count) {
        size_t bytes = (count * sizeof(T) + 255) & ~size_t(255);
        T* p = reinterpret_cast<T*>(base + used);
        used += bytes;
        return p;
    }
    static size_t round(size_t bytes) { return (bytes + 255) & ~size_t(255); }
};

struct NttTables;  // ntt.cu

struct DeviceContext {
    int device = -1;
    int num_sms = 0;
    cudaStream_t stream = nullptr;   // default work stream
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t ev_a = nullptr, ev_b = nullptr, ev_c = nullptr;
    cudaEvent_t scratch_done = nullptr;  // last work that used `scratch`
    cudaEvent_t phase[9] = {};            // MSM phase boundaries (timing)
    cudaStream_t aux_stream = nullptr;    // pipelined host MSM: sorts beside the accumulates
    cudaEvent_t batch_ev[12] = {};        // pipelined host MSM: per batch scalars landed, points landed, keys sorted
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    void* pinned = nullptr;          // small pinned host staging (results)
    size_t pinned_bytes = 0;
    NttTables* ntt = nullptr;
    cudaStream_t set_stream[8] = {};  // MSMs sharing one sort: one stream per point set (created on first use)
    std::mutex mu;                   // one call at a time per device context
};

// Lazily created context of `device` (-1 = the calling thread's current device).
// Makes `device` current on the calling thread.
int get_context(int device, DeviceContext** out);
// A private context on `device` (its own streams, scratch and lock), for work
// that runs beside calls on the device's shared context; freed by
// destroy_context after its streams drain.
int create_context(int device, DeviceContext** out);
void destroy_context(DeviceContext* ctx);
// Frees the NTT tables cached in a context (ntt.cu).
void release_ntt_tables(DeviceContext* ctx);
// Ensure the scratch arena holds at least `bytes` (synchronises on growth).
int ensure_scratch(DeviceContext* ctx, size_t bytes);
int ensure_pinned(DeviceContext* ctx, size_t bytes);
// Order a call's work on `st` after the previous user of the scratch arena
// (which may have run on another stream), and mark the end of its use.
int scratch_begin(DeviceContext* ctx, cudaStream_t st);
// The per-set streams of a context (msm_shared_scalars_run).
int ensure_set_streams(DeviceContext* ctx);
int scratch_end(DeviceContext* ctx, cudaStream_t st);

// per-thread statistics of the last MSM
struct MsmStats {
    int kernel_launches = 0;
    float accumulate_ms = 0.f;
    float total_device_ms = 0.f;
    int window_bits = 0;
    int num_windows = 0;
    long long bucket_adds = 0;
    float phase_ms[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    long long ba_pairs = 0;  // affine pair additions of the batch-affine rounds
    long long ba_left = 0;   // elements left after them for the XYZZ accumulation
};
MsmStats& msm_stats();

// Precomputed window tables of fixed G1 bases (msm.cu): 2^(c j) P_i for j < W
// at index j n + i; the MSM of scalars[0, hi - lo) against bases [lo, hi).
void g1_window_tables_shape(size_t n, int* c, int* W);
int g1_window_tables_build(int device, cudaStream_t st, const void* d_points, size_t n, int c, int W, void* d_out);
// Several MSMs (G1 or G2 point sets) over the same device scalars with one
// shared counting sort (msm.cu), in the scratch of `ctx`; outs[k]: 64 or 128
// host bytes.
int msm_shared_scalars_run(DeviceContext* ctx, cudaStream_t st, const void* d_scalars, size_t n, int n_sets, const void* const* d_points,
                           const int* is_g2, const uint32_t* idx_range, uint64_t* const* outs, float* set_ms);
int g1_window_tables_msm(int device, cudaStream_t st, const void* tables, size_t n_total, int c, int W, size_t lo, size_t hi,
                         const void* d_scalars, uint64_t* out_affine);

}  // namespace zk
