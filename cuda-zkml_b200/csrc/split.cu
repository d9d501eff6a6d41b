// split.cu -- a Groth16 proof split over several devices (the reference proves
// on device 0 only: Groth16Prover::prove, src/prover/groth16.cu:655-920).
//
// Every rank holds the whole proving key and R1CS on its own device and gets
// the same proof bytes as the one-device prover:
//   1. each rank uploads a quarter of its slice of the witness at a time, and
//      each round's slices are all-gathered while the next round is uploaded;
//   2. rank j computes constraint rows [j m, (j + 1) m) of A w, B w, C w
//      (m = n / N) and checks them (R1CS::verify_witness, src/prover/
//      circuit.cuh:93-124); the first failing row is an all-reduce MIN, read at
//      the end, so every rank fails alike;
//   3. the witness MSMs (A, B2, B1, L over rank j's slice of the witness, one
//      shared sort) run from a host thread on the key's private device context,
//      beside steps 4-5;
//   4. compute_h (groth16.cu:263-390) with every transform split over the
//      ranks: a size-m transform on each rank, one all-to-all, and the
//      cross-rank N-point step (ntt_cross_run).  The all-to-alls are grouped
//      point-to-point copies whose send and receive blocks are contiguous by
//      construction (a gather kernel writes the first one's send layout), so no
//      layout copy surrounds them; they run one polynomial at a time on a
//      second stream, so one polynomial travels while another is transformed;
//   5. rank j's H MSM over its own coefficients of h (h_msm_blocks);
//   6. the partial sums (384 B per rank) are all-gathered and every rank folds
//      them and assembles the proof (zk_groth16_assemble_parts).
// Communicators: NCCL (loaded at run time; one process per GPU, or one process
// driving several GPUs with a host thread each), or ranks as host threads
// sharing one device (copies on the device, host barriers) for testing the
// split where only one GPU is at hand.  No kernel waits on another rank: every
// exchange is an NCCL operation or a stream-ordered copy into the receiving
// device's own memory, and no kernel reads a peer's memory.
#include "prover.hpp"

#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>

// ------------------------------------------------------------------ communicators
namespace zk {
namespace split {

// One exchange of an all-to-all: this rank sends `bytes` at `send` to `peer`
// and receives `bytes` from `peer` into `recv` (both device memory).
struct Xfer {
    int peer;
    const void* send;
    void* recv;
    size_t bytes;
};

struct Comm {
    int nranks = 1, rank = 0, device = 0;
    virtual ~Comm() {}
    // recv gets nranks blocks of `bytes` in rank order; send may be recv + rank * bytes
    virtual int all_gather(const void* send, void* recv, size_t bytes, cudaStream_t st) = 0;
    // elementwise minimum over the ranks of `count` u64, in place
    virtual int all_reduce_min(uint64_t* buf, size_t count, cudaStream_t st) = 0;
    // grouped point-to-point copies; every rank lists one Xfer per peer (itself included)
    virtual int exchange(const Xfer* x, int count, cudaStream_t st) = 0;
    virtual int abort() = 0;
};

// ---------------------------------------------------------------- NCCL, loaded at run time
struct NcclApi {
    bool loaded = false;
    std::string err;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommInitAll)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

// libnccl.so.2 (ZKML_NCCL_LIB overrides): the copy already loaded in the
// process, if any (a framework's), else the system's.
static NcclApi& nccl() {
    static std::once_flag once;
    static NcclApi api;
    std::call_once(once, [] {
        const char* name = getenv("ZKML_NCCL_LIB");
        void* h = dlopen(name && *name ? name : "libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            api.err = std::string("cannot load NCCL: ") + dlerror();
            return;
        }
#define ZK_NCCL_SYM(field, sym)                                     \
    api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, sym)); \
    if (!api.field) {                                               \
        api.err = std::string("NCCL lacks ") + sym;                 \
        return;                                                     \
    }
        ZK_NCCL_SYM(GetUniqueId, "ncclGetUniqueId")
        ZK_NCCL_SYM(CommInitRank, "ncclCommInitRank")
        ZK_NCCL_SYM(CommInitAll, "ncclCommInitAll")
        ZK_NCCL_SYM(CommDestroy, "ncclCommDestroy")
        ZK_NCCL_SYM(CommAbort, "ncclCommAbort")
        ZK_NCCL_SYM(AllGather, "ncclAllGather")
        ZK_NCCL_SYM(AllReduce, "ncclAllReduce")
        ZK_NCCL_SYM(Send, "ncclSend")
        ZK_NCCL_SYM(Recv, "ncclRecv")
        ZK_NCCL_SYM(GroupStart, "ncclGroupStart")
        ZK_NCCL_SYM(GroupEnd, "ncclGroupEnd")
        ZK_NCCL_SYM(GetErrorString, "ncclGetErrorString")
#undef ZK_NCCL_SYM
        api.loaded = true;
    });
    return api;
}

static int nccl_ready() {
    NcclApi& a = nccl();
    if (!a.loaded) {
        set_error("%s", a.err.c_str());
        return ZK_ERR_NODEV;
    }
    return ZK_OK;
}

#define ZK_TRY_NCCL(call)                                                                             \
    do {                                                                                              \
        ncclResult_t r_ = (call);                                                                     \
        if (r_ != ncclSuccess) {                                                                      \
            ::zk::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call, nccl().GetErrorString(r_)); \
            return ZK_ERR_CUDA;                                                                       \
        }                                                                                             \
    } while (0)

struct NcclComm : Comm {
    std::atomic<ncclComm_t> c{nullptr};  // cleared by abort(), possibly from a watchdog thread
    ~NcclComm() override {
        ncclComm_t t = c.exchange(nullptr);
        if (t) nccl().CommDestroy(t);
    }
    int all_gather(const void* send, void* recv, size_t bytes, cudaStream_t st) override {
        ZK_TRY_NCCL(nccl().AllGather(send, recv, bytes, ncclUint8, c, st));
        return ZK_OK;
    }
    int all_reduce_min(uint64_t* buf, size_t count, cudaStream_t st) override {
        ZK_TRY_NCCL(nccl().AllReduce(buf, buf, count, ncclUint64, ncclMin, c, st));
        return ZK_OK;
    }
    int exchange(const Xfer* x, int count, cudaStream_t st) override {
        ZK_TRY_NCCL(nccl().GroupStart());
        ncclResult_t bad = ncclSuccess;
        for (int i = 0; i < count && bad == ncclSuccess; i++) {
            bad = nccl().Send(x[i].send, x[i].bytes, ncclUint8, x[i].peer, c, st);
            if (bad == ncclSuccess) bad = nccl().Recv(x[i].recv, x[i].bytes, ncclUint8, x[i].peer, c, st);
        }
        ZK_TRY_NCCL(nccl().GroupEnd());  // closes the group on every path
        ZK_TRY_NCCL(bad);
        return ZK_OK;
    }
    int abort() override {
        ncclComm_t t = c.exchange(nullptr);
        if (t) ZK_TRY_NCCL(nccl().CommAbort(t));
        return ZK_OK;
    }
};

// ---------------------------------------------------------------- ranks as threads on one device
// Each collective: every rank records a "ready" event after the work that
// produced its buffers and publishes them; after a host barrier each rank
// copies what it receives on its own stream (after the senders' ready events)
// and records "done"; after a second barrier it orders its stream after every
// rank's done (its send buffers are then free to change), and a third barrier
// keeps the events from being recorded again before everyone has waited on
// them.  Barriers give up after a time limit or an abort.
struct LocalShared {
    int nranks = 0;
    double timeout_s = 300.0;
    std::mutex mu;
    std::condition_variable cv;
    int arrived = 0;
    uint64_t generation = 0;
    bool aborted = false;
    std::vector<const void*> ptr;
    std::vector<const Xfer*> xf;
    std::vector<int> nx;
    std::vector<cudaEvent_t> ready, done;
    std::atomic<int> refs{0};

    bool barrier() {
        std::unique_lock<std::mutex> lk(mu);
        if (aborted) return false;
        const uint64_t gen = generation;
        if (++arrived == nranks) {
            arrived = 0;
            generation++;
            cv.notify_all();
            return true;
        }
        const bool ok = cv.wait_for(lk, std::chrono::duration<double>(timeout_s), [&] { return aborted || generation != gen; });
        return ok && !aborted;
    }
    void abort() {
        std::lock_guard<std::mutex> lk(mu);
        aborted = true;
        cv.notify_all();
    }
};

__global__ void min_u64_kernel(uint64_t* __restrict__ out, const uint64_t* __restrict__ all, size_t count, int nranks) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
        uint64_t v = all[i];
        for (int r = 1; r < nranks; r++) v = min(v, all[(size_t)r * count + i]);
        out[i] = v;
    }
}

struct LocalComm : Comm {
    LocalShared* sh = nullptr;
    uint64_t* tmp = nullptr;  // all_reduce_min staging
    size_t tmp_count = 0;
    ~LocalComm() override {
        if (tmp) cudaFree(tmp);
        if (sh && --sh->refs == 0) {
            for (auto e : sh->ready) cudaEventDestroy(e);
            for (auto e : sh->done) cudaEventDestroy(e);
            delete sh;
        }
    }
    int fail_barrier() {
        set_error("split prove: ranks-as-threads barrier %s", sh->aborted ? "aborted" : "timed out");
        return ZK_ERR_CUDA;
    }
    // phase 1: publish + barrier; phase 2: copies (caller) + done + barrier + wait + barrier
    int finish(cudaStream_t st) {
        ZK_TRY_CUDA(cudaEventRecord(sh->done[rank], st));
        if (!sh->barrier()) return fail_barrier();
        for (int j = 0; j < nranks; j++) ZK_TRY_CUDA(cudaStreamWaitEvent(st, sh->done[j], 0));
        if (!sh->barrier()) return fail_barrier();
        return ZK_OK;
    }
    int all_gather(const void* send, void* recv, size_t bytes, cudaStream_t st) override {
        ZK_TRY_CUDA(cudaEventRecord(sh->ready[rank], st));
        sh->ptr[rank] = send;
        if (!sh->barrier()) return fail_barrier();
        for (int j = 0; j < nranks; j++) {
            ZK_TRY_CUDA(cudaStreamWaitEvent(st, sh->ready[j], 0));
            if ((char*)recv + (size_t)j * bytes != sh->ptr[j])
                ZK_TRY_CUDA(cudaMemcpyAsync((char*)recv + (size_t)j * bytes, sh->ptr[j], bytes, cudaMemcpyDeviceToDevice, st));
        }
        return finish(st);
    }
    int all_reduce_min(uint64_t* buf, size_t count, cudaStream_t st) override {
        if (tmp_count < count * nranks) {
            if (tmp) cudaFree(tmp);
            tmp = nullptr;
            tmp_count = 0;
            ZK_TRY_CUDA(cudaMalloc(&tmp, count * nranks * 8));
            tmp_count = count * nranks;
        }
        ZK_TRY(all_gather(buf, tmp, count * 8, st));
        min_u64_kernel<<<1, 256, 0, st>>>(buf, tmp, count, nranks);
        ZK_TRY_CUDA(cudaGetLastError());
        return ZK_OK;
    }
    int exchange(const Xfer* x, int count, cudaStream_t st) override {
        ZK_TRY_CUDA(cudaEventRecord(sh->ready[rank], st));
        sh->xf[rank] = x;
        sh->nx[rank] = count;
        if (!sh->barrier()) return fail_barrier();
        for (int i = 0; i < count; i++) {
            const int j = x[i].peer;
            // the peer's entry addressed to this rank, k-th of its kind (several per peer are matched in order)
            int kth = 0;
            for (int p = 0; p < i; p++) kth += x[p].peer == j;
            const Xfer* src = nullptr;
            for (int p = 0, seen = 0; p < sh->nx[j]; p++)
                if (sh->xf[j][p].peer == rank && seen++ == kth) { src = &sh->xf[j][p]; break; }
            if (!src || src->bytes != x[i].bytes) {
                set_error("split prove: unmatched exchange between ranks %d and %d", rank, j);
                sh->abort();
                return ZK_ERR_INVALID;
            }
            ZK_TRY_CUDA(cudaStreamWaitEvent(st, sh->ready[j], 0));
            ZK_TRY_CUDA(cudaMemcpyAsync(x[i].recv, src->send, x[i].bytes, cudaMemcpyDeviceToDevice, st));
        }
        return finish(st);
    }
    int abort() override {
        sh->abort();
        return ZK_OK;
    }
};

}  // namespace split
}  // namespace zk

struct zk_comm {
    zk::split::Comm* c = nullptr;
};

// ------------------------------------------------------------------ the split prove
namespace zk {
namespace split {

static constexpr int kSumWords = 48;  // A (8) | B2 (16) | L (8) | H (8) | B1 (8)
static constexpr int kRecWords = 49;  // the sums, then the rank's status (0: its part succeeded)
static constexpr int kWitnessChunks = 4;  // upload rounds of the witness, each all-gathered behind the next

// dst[k][j][t] = src[k][j + N t]: rows of this rank's block regrouped by
// residue mod N, the send layout of the first all-to-all (to the "cyclic"
// layout, where rank j holds global rows j + N t).
__global__ void cyclic_gather_kernel(const Fr* __restrict__ src, Fr* __restrict__ dst, uint64_t m, int log_parts) {
    const uint64_t q = m >> log_parts;
    const uint64_t total = 3 * m;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t k = i / m, r = i - k * m;  // destination index within vector k
        const uint64_t j = r / q, t = r - j * q;
        Fr v;
        fload_nc(v, src + k * m + j + (t << log_parts));
        fstore(dst + i, v);
    }
}

struct State {
    int device = -1, nranks = 0, rank = 0;
    uint64_t n = 0, m = 0, q = 0;
    size_t cw = 0;  // witness rows per rank and upload round (padded: N kWitnessChunks cw >= witness rows)
    cudaStream_t st = nullptr;
    cudaStream_t cst = nullptr;  // the all-to-alls of compute_h, beside the transforms on st
    Fr* w = nullptr;    // kWitnessChunks * nranks * cw
    Fr* p[3] = {};      // three buffers of 3 m
    unsigned long long* bad = nullptr;
    uint64_t* rec = nullptr;          // nranks * kRecWords
    unsigned long long* h_bad = nullptr;  // pinned
    uint64_t* h_rec = nullptr;            // pinned, nranks * kRecWords
    cudaEvent_t ev[16] = {};
    cudaEvent_t dep[16] = {};  // ordering between st and cst (no timing)
    cudaEvent_t xev[20] = {};  // begin and end of each all-to-all on cst
    std::vector<Xfer> xf;
    ~State() {
        if (device >= 0) cudaSetDevice(device);
        if (st) cudaStreamSynchronize(st);
        if (cst) cudaStreamSynchronize(cst);
        cudaFree(w);
        for (auto b : p) cudaFree(b);
        cudaFree(bad);
        cudaFree(rec);
        cudaFreeHost(h_bad);
        cudaFreeHost(h_rec);
        for (auto e : ev)
            if (e) cudaEventDestroy(e);
        for (auto e : dep)
            if (e) cudaEventDestroy(e);
        for (auto e : xev)
            if (e) cudaEventDestroy(e);
        if (st) cudaStreamDestroy(st);
        if (cst) cudaStreamDestroy(cst);
    }
};

static int get_state(zk_groth16_pk* pk, const R1cs& R, int nranks, int rank, State** out) {
    std::lock_guard<std::mutex> lock(pk->h_mu);
    auto it = pk->split.find({nranks, rank});
    if (it != pk->split.end()) {
        *out = it->second;
        return ZK_OK;
    }
    State* s = new State();
    auto fail = [&](int rc) {
        delete s;
        return rc;
    };
    s->device = pk->device;
    s->nranks = nranks;
    s->rank = rank;
    s->n = R.n;
    s->m = R.n / (uint64_t)nranks;
    s->q = s->m / (uint64_t)nranks;
    s->cw = ((size_t)R.m + (size_t)nranks * kWitnessChunks - 1) / ((size_t)nranks * kWitnessChunks);
#define ZK_S(call)                                                                                           \
    do {                                                                                                     \
        cudaError_t e_ = (call);                                                                             \
        if (e_ != cudaSuccess) {                                                                             \
            set_error("split prove buffers: %s: %s", #call, cudaGetErrorString(e_));                        \
            return fail(e_ == cudaErrorMemoryAllocation ? ZK_ERR_NOMEM : ZK_ERR_CUDA);                      \
        }                                                                                                    \
    } while (0)
    ZK_S(cudaSetDevice(pk->device));
    ZK_S(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
    ZK_S(cudaStreamCreateWithFlags(&s->cst, cudaStreamNonBlocking));
    ZK_S(cudaMalloc(&s->w, s->cw * nranks * kWitnessChunks * 32));
    for (auto& b : s->p) ZK_S(cudaMalloc(&b, 3 * s->m * 32));
    ZK_S(cudaMalloc(&s->bad, 8));
    ZK_S(cudaMalloc(&s->rec, (size_t)nranks * kRecWords * 8));
    ZK_S(cudaMallocHost(&s->h_bad, 8));
    ZK_S(cudaMallocHost(&s->h_rec, (size_t)nranks * kRecWords * 8));
    for (auto& e : s->ev) ZK_S(cudaEventCreate(&e));
    for (auto& e : s->dep) ZK_S(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    for (auto& e : s->xev) ZK_S(cudaEventCreate(&e));
#undef ZK_S
    pk->split[{nranks, rank}] = s;
    *out = s;
    return ZK_OK;
}

// per-thread statistics of the last split prove
static thread_local zk_split_stats g_stats;

static float ev_ms(cudaEvent_t a, cudaEvent_t b) {
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    return ms;
}

// An all-to-all of one vector of m values on the exchange stream: block j (q
// values) goes to rank j, and the block from rank j lands at block j.
static int all_to_all(Comm* comm, State* S, const Fr* send, Fr* recv) {
    S->xf.clear();
    for (int j = 0; j < S->nranks; j++) S->xf.push_back({j, send + (uint64_t)j * S->q, recv + (uint64_t)j * S->q, S->q * 32});
    return comm->exchange(S->xf.data(), (int)S->xf.size(), S->cst);
}

// The all-to-alls of compute_h run one polynomial at a time on the exchange
// stream, each after the transform that produced its vector and before the
// transform that consumes it, so that one polynomial crosses NVLink while
// another is transformed.  Every rank issues them in the same order.
struct Pipe {
    State* S;
    Comm* comm;
    int nx = 0;  // all-to-alls issued (timing events xev[2 i], xev[2 i + 1])
    int nd = 0;  // ordering events used
    int xchg(cudaEvent_t after, const Fr* send, Fr* recv, cudaEvent_t* done) {
        ZK_TRY_CUDA(cudaStreamWaitEvent(S->cst, after, 0));
        ZK_TRY_CUDA(cudaEventRecord(S->xev[2 * nx], S->cst));
        ZK_TRY(all_to_all(comm, S, send, recv));
        ZK_TRY_CUDA(cudaEventRecord(S->xev[2 * nx + 1], S->cst));
        nx++;
        *done = S->xev[2 * nx - 1];
        return ZK_OK;
    }
    int mark(cudaStream_t st, cudaEvent_t* e) {
        *e = S->dep[nd++];
        ZK_TRY_CUDA(cudaEventRecord(*e, st));
        return ZK_OK;
    }
    float exchange_ms() const {
        float t = 0;
        for (int i = 0; i < nx; i++) {
            float ms = 0;
            cudaEventElapsedTime(&ms, S->xev[2 * i], S->xev[2 * i + 1]);
            t += ms;
        }
        return t;
    }
};

static int prove_split(zk_groth16_pk* pk, const R1cs& R, Comm* comm, const void* h_witness, const void* r, const void* s, void* proof256,
                       void* points) {
    auto t_start = std::chrono::steady_clock::now();
    zk_split_stats& stats = g_stats;
    std::memset(&stats, 0, sizeof stats);
    const int N = comm->nranks, me = comm->rank;
    stats.nranks = N;
    stats.rank = me;
    int log_parts = 0;
    while ((1 << log_parts) < N) log_parts++;
    if (R.m != pk->m || R.num_public != pk->num_public || (uint64_t)pk->num_constraints != R.n) {
        set_error("split prove: proving key (m %d, public %d, n %d) does not match the circuit (m %d, public %d, n %llu)", pk->m,
                  pk->num_public, pk->num_constraints, R.m, R.num_public, (unsigned long long)R.n);
        return ZK_ERR_INVALID;
    }
    if ((1 << log_parts) != N || log_parts > 3 || 2 * log_parts > R.log_n) {
        set_error("split prove: %d ranks (a power of two up to 8, with ranks^2 <= %llu)", N, (unsigned long long)R.n);
        return ZK_ERR_RANGE;
    }
    if (pk->device != comm->device) {
        set_error("split prove: key on device %d, communicator rank on device %d", pk->device, comm->device);
        return ZK_ERR_INVALID;
    }
    DeviceContext* ctx;
    ZK_TRY(get_context(pk->device, &ctx));
    ZK_TRY(ensure_witness_context(pk));
    State* S;
    ZK_TRY(get_state(pk, R, N, me, &S));
    cudaStream_t st = S->st;
    const uint64_t m = S->m, L = (uint64_t)R.log_n;
    cudaEvent_t* ev = S->ev;
    Fr *P0 = S->p[0], *P1 = S->p[1], *P2 = S->p[2];
    zkh::Fe g;
    ZK_TRY(zk_compute_h_coset_shift(R.log_n, g.v));

    // 1. witness: kWitnessChunks rounds; in round c rank r uploads global rows
    //    [(c N + r) cw, (c N + r + 1) cw) and the round's N chunks are
    //    all-gathered on the exchange stream while the next round's chunk crosses
    //    PCIe on the work stream
    Pipe pp{S, comm};
    ZK_TRY_CUDA(cudaEventRecord(ev[0], st));
    const size_t cw = S->cw;
    for (int c = 0; c < kWitnessChunks; c++) {
        const size_t at = ((size_t)c * N + me) * cw;
        const size_t lo_c = std::min((size_t)R.m, at), hi_c = std::min((size_t)R.m, at + cw);
        if (hi_c > lo_c)
            ZK_TRY_CUDA(cudaMemcpyAsync(S->w + at, (const uint8_t*)h_witness + lo_c * 32, (hi_c - lo_c) * 32, cudaMemcpyHostToDevice, st));
        if (cw > hi_c - lo_c) ZK_TRY_CUDA(cudaMemsetAsync(S->w + at + (hi_c - lo_c), 0, (cw - (hi_c - lo_c)) * 32, st));
        cudaEvent_t up;
        ZK_TRY(pp.mark(st, &up));
        ZK_TRY_CUDA(cudaStreamWaitEvent(S->cst, up, 0));
        ZK_TRY(comm->all_gather(S->w + at, S->w + (size_t)c * N * cw, cw * 32, S->cst));
    }
    {
        cudaEvent_t ag;
        ZK_TRY(pp.mark(S->cst, &ag));
        ZK_TRY_CUDA(cudaStreamWaitEvent(st, ag, 0));
    }
    ZK_TRY_CUDA(cudaEventRecord(ev[1], st));

    // 3. the witness MSMs over an equal slice of the witness, from a host thread
    //    on the key's private context, after the all-gather
    const size_t a_lo = (size_t)R.m * me / N, a_hi = (size_t)R.m * (me + 1) / N;
    uint64_t sums[kRecWords] = {};  // the rank's partial sums and its status word
    float set_ms[4] = {0, 0, 0, 0}, wit_all = 0;
    int wit_rc = ZK_OK;
    std::string wit_err;
    struct Joiner {
        std::thread t;
        ~Joiner() {
            if (t.joinable()) t.join();
        }
    } worker;
    DeviceContext* wctx = pk->wctx;
    ZK_TRY_CUDA(cudaStreamWaitEvent(wctx->stream, ev[1], 0));
    worker.t = std::thread([&, wctx]() {
        if (cudaSetDevice(wctx->device) != cudaSuccess) {
            wit_rc = ZK_ERR_CUDA;
            wit_err = "witness MSMs: cudaSetDevice failed";
            return;
        }
        wit_rc = witness_msms(pk, wctx, wctx->stream, S->w, a_lo, a_hi, sums, sums + 8, sums + 40, sums + 24, set_ms, &wit_all);
        if (wit_rc != ZK_OK) wit_err = zk_last_error();
    });

    // 2. rows of the matvec and their check (read at the end)
    const uint64_t lo = m * me;
    ZK_TRY(r1cs_matvec_rows(R, st, S->w, lo, lo + m, P0, ctx->num_sms));
    const bool check = witness_check_enabled();
    ZK_TRY_CUDA(cudaMemsetAsync(S->bad, 0xff, 8, st));
    if (check) enqueue_hadamard_check(st, P0, P0 + m, P0 + 2 * m, m, lo, S->bad, ctx->num_sms);
    ZK_TRY(comm->all_reduce_min((uint64_t*)S->bad, 1, st));
    ZK_TRY_CUDA(cudaMemcpyAsync(S->h_bad, S->bad, 8, cudaMemcpyDeviceToHost, st));
    ZK_TRY_CUDA(cudaEventRecord(ev[2], st));

    // 4. compute_h, every transform split over the ranks; the all-to-alls on
    //    the exchange stream, one polynomial at a time (Pipe)
    {
        const unsigned grid = (unsigned)std::min<uint64_t>((3 * m + 255) / 256, (uint64_t)ctx->num_sms * 16);
        cyclic_gather_kernel<<<grid, 256, 0, st>>>(P0, P2, m, log_parts);
        ZK_TRY_CUDA(cudaGetLastError());
    }
    cudaEvent_t e_rows, e_in[3], e_x[3], e_out[3], e_co[3], e_ev[3], e_h, e_hx;
    ZK_TRY(pp.mark(st, &e_rows));
    for (int k = 0; k < 3; k++)  // evaluations, cyclic
        ZK_TRY(pp.xchg(e_rows, P2 + k * m, P1 + k * m, &e_in[k]));
    for (int k = 0; k < 3; k++) {  // the size-m INTT of each polynomial as its values land
        ZK_TRY_CUDA(cudaStreamWaitEvent(st, e_in[k], 0));
        ZK_TRY(zk_ntt_device(pk->device, st, P1 + k * m, P1 + k * m, (int)L - log_parts, 1, nullptr));
        ZK_TRY(pp.mark(st, &e_x[k]));
        ZK_TRY(pp.xchg(e_x[k], P1 + k * m, P2 + k * m, &e_out[k]));
    }
    for (int k = 0; k < 3; k++) {  // coefficients n^-1 g^i, blocks; then toward the coset evaluations
        ZK_TRY_CUDA(cudaStreamWaitEvent(st, e_out[k], 0));
        ZK_TRY(zk_ntt_cross_device(pk->device, st, P1 + k * m, P2 + k * m, (int)L, log_parts, me, 1, 0, g.v, 0));
        ZK_TRY(zk_ntt_cross_device(pk->device, st, P0 + k * m, P1 + k * m, (int)L, log_parts, me, 0, 1, nullptr, 0));
        ZK_TRY(pp.mark(st, &e_co[k]));
        ZK_TRY(pp.xchg(e_co[k], P0 + k * m, P2 + k * m, &e_ev[k]));  // coset evaluations, cyclic
    }
    for (int k = 0; k < 3; k++) {
        ZK_TRY_CUDA(cudaStreamWaitEvent(st, e_ev[k], 0));
        ZK_TRY(zk_ntt_device(pk->device, st, P2 + k * m, P2 + k * m, (int)L - log_parts, 0, nullptr));
    }
    ZK_TRY(zk_compute_h_pointwise_device(pk->device, st, P1, P2, P2 + m, P2 + 2 * m, (int)L, m));
    ZK_TRY(zk_ntt_device(pk->device, st, P1, P1, (int)L - log_parts, 1, nullptr));
    ZK_TRY(pp.mark(st, &e_h));
    ZK_TRY(pp.xchg(e_h, P1, P0, &e_hx));
    ZK_TRY_CUDA(cudaStreamWaitEvent(st, e_hx, 0));
    ZK_TRY(zk_ntt_cross_device(pk->device, st, P1, P0, (int)L, log_parts, me, 1, 0, g.v, 1));  // h, blocks, n^-1 g^-i
    ZK_TRY_CUDA(cudaEventRecord(ev[11], st));

    // 5. this rank's H MSM (synchronises the stream)
    uint64_t h_sum[8] = {0};
    if (pk->n_h > 0) ZK_TRY(h_msm_blocks(pk, st, P1, log_parts, me, h_sum));
    ZK_TRY_CUDA(cudaEventRecord(ev[12], st));
    auto t_wait = std::chrono::steady_clock::now();
    worker.t.join();
    stats.witness_wait_ms = std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - t_wait).count();
    std::memcpy(sums + 32, h_sum, 64);
    // a failed witness MSM still takes part in the sums' all-gather (every rank
    // makes the same collective calls) and marks its record, so every rank
    // fails the proof alike
    sums[kSumWords] = wit_rc == ZK_OK ? 0 : 1;

    // 6. partial sums to every rank
    ZK_TRY_CUDA(cudaMemcpyAsync(S->rec + (size_t)me * kRecWords, sums, kRecWords * 8, cudaMemcpyHostToDevice, st));
    ZK_TRY(comm->all_gather(S->rec + (size_t)me * kRecWords, S->rec, kRecWords * 8, st));
    ZK_TRY_CUDA(cudaMemcpyAsync(S->h_rec, S->rec, (size_t)N * kRecWords * 8, cudaMemcpyDeviceToHost, st));
    ZK_TRY_CUDA(cudaEventRecord(ev[13], st));
    ZK_TRY_CUDA(cudaEventSynchronize(ev[13]));
    for (int j = 0; j < N; j++)
        if (S->h_rec[(size_t)j * kRecWords + kSumWords] != 0) {
            if (j == me) set_error("%s", wit_err.c_str());
            else set_error("split prove: the witness MSMs of rank %d failed", j);
            return j == me ? wit_rc : ZK_ERR_CUDA;
        }
    if (check && *S->h_bad != ~0ull) {
        set_error("[Prove] Witness does not satisfy R1CS constraints (constraint %llu failed)", *S->h_bad);
        return ZK_ERR_INVALID;
    }
    auto t_asm = std::chrono::steady_clock::now();
    std::vector<uint64_t> parts((size_t)N * kSumWords);
    for (int j = 0; j < N; j++) std::memcpy(&parts[(size_t)j * kSumWords], S->h_rec + (size_t)j * kRecWords, kSumWords * 8);
    ZK_TRY(zk_groth16_assemble_parts(pk, r, s, parts.data(), N, proof256, points));
    auto t_end = std::chrono::steady_clock::now();

    stats.witness_ms = ev_ms(ev[0], ev[1]);
    stats.matvec_ms = ev_ms(ev[1], ev[2]);
    stats.compute_h_ms = ev_ms(ev[2], ev[11]);
    stats.all_to_all_ms = pp.exchange_ms();  // on the exchange stream, overlapping the transforms
    stats.h_msm_ms = ev_ms(ev[11], ev[12]);
    stats.witness_msms_ms = wit_all;
    stats.gather_ms = ev_ms(ev[12], ev[13]);
    stats.assemble_ms = std::chrono::duration<float, std::milli>(t_end - t_asm).count();
    stats.total_ms = std::chrono::duration<float, std::milli>(t_end - t_start).count();
    return ZK_OK;
}

}  // namespace split

void destroy_split_states(zk_groth16_pk* pk) {
    for (auto& kv : pk->split) delete kv.second;
    pk->split.clear();
}

}  // namespace zk

// ================================================================== C ABI (split prove)
using namespace zk;

extern "C" int zk_comm_unique_id(void* id128) {
    clear_error();
    if (!id128) return ZK_ERR_INVALID;
    ZK_TRY(split::nccl_ready());
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId layout");
    ncclUniqueId id;
    ncclResult_t r = split::nccl().GetUniqueId(&id);
    if (r != ncclSuccess) {
        set_error("ncclGetUniqueId: %s", split::nccl().GetErrorString(r));
        return ZK_ERR_CUDA;
    }
    std::memcpy(id128, &id, 128);
    return ZK_OK;
}

extern "C" int zk_comm_init_rank(int device, const void* id128, int nranks, int rank, zk_comm** out) {
    clear_error();
    if (!id128 || !out || nranks < 1 || rank < 0 || rank >= nranks) return ZK_ERR_INVALID;
    *out = nullptr;
    ZK_TRY(split::nccl_ready());
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    ncclUniqueId id;
    std::memcpy(&id, id128, 128);
    auto* c = new split::NcclComm();
    c->nranks = nranks;
    c->rank = rank;
    c->device = ctx->device;
    ncclComm_t nc = nullptr;
    ncclResult_t r = split::nccl().CommInitRank(&nc, nranks, id, rank);
    if (r != ncclSuccess) {
        set_error("ncclCommInitRank: %s", split::nccl().GetErrorString(r));
        delete c;
        return ZK_ERR_CUDA;
    }
    c->c = nc;
    *out = new zk_comm{c};
    return ZK_OK;
}

extern "C" int zk_comm_init_all(const int* devices, int ndev, zk_comm** comms) {
    clear_error();
    if (!devices || !comms || ndev < 1 || ndev > 64) return ZK_ERR_INVALID;
    for (int i = 0; i < ndev; i++) comms[i] = nullptr;
    ZK_TRY(split::nccl_ready());
    for (int i = 0; i < ndev; i++) {
        DeviceContext* ctx;
        ZK_TRY(get_context(devices[i], &ctx));
    }
    std::vector<ncclComm_t> cs((size_t)ndev);
    ncclResult_t r = split::nccl().CommInitAll(cs.data(), ndev, devices);
    if (r != ncclSuccess) {
        set_error("ncclCommInitAll: %s", split::nccl().GetErrorString(r));
        return ZK_ERR_CUDA;
    }
    for (int i = 0; i < ndev; i++) {
        auto* c = new split::NcclComm();
        c->nranks = ndev;
        c->rank = i;
        c->device = devices[i];
        c->c = cs[(size_t)i];
        comms[i] = new zk_comm{c};
    }
    return ZK_OK;
}

extern "C" int zk_comm_init_local(int device, int nranks, zk_comm** comms) {
    clear_error();
    if (!comms || nranks < 1 || nranks > 64) return ZK_ERR_INVALID;
    for (int i = 0; i < nranks; i++) comms[i] = nullptr;
    DeviceContext* ctx;
    ZK_TRY(get_context(device, &ctx));
    auto* sh = new split::LocalShared();
    sh->nranks = nranks;
    sh->ptr.assign((size_t)nranks, nullptr);
    sh->xf.assign((size_t)nranks, nullptr);
    sh->nx.assign((size_t)nranks, 0);
    sh->ready.assign((size_t)nranks, nullptr);
    sh->done.assign((size_t)nranks, nullptr);
    for (int i = 0; i < nranks; i++) {
        if (cudaEventCreateWithFlags(&sh->ready[i], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&sh->done[i], cudaEventDisableTiming) != cudaSuccess) {
            set_error("local communicator: event creation failed");
            for (auto e : sh->ready) if (e) cudaEventDestroy(e);
            for (auto e : sh->done) if (e) cudaEventDestroy(e);
            delete sh;
            return ZK_ERR_CUDA;
        }
    }
    for (int i = 0; i < nranks; i++) {
        auto* c = new split::LocalComm();
        c->nranks = nranks;
        c->rank = i;
        c->device = ctx->device;
        c->sh = sh;
        sh->refs++;
        comms[i] = new zk_comm{c};
    }
    return ZK_OK;
}

extern "C" int zk_comm_abort(zk_comm* comm) {
    clear_error();
    if (!comm || !comm->c) return ZK_ERR_INVALID;
    return comm->c->abort();
}

extern "C" void zk_comm_destroy(zk_comm* comm) {
    if (!comm) return;
    delete comm->c;
    delete comm;
}

extern "C" int zk_groth16_prove_split(zk_groth16_pk* pk, const zk_r1cs* r1cs, zk_comm* comm, const void* h_witness, const void* r,
                                      const void* s, void* proof256, void* points) {
    clear_error();
    if (!pk || !r1cs || !comm || !comm->c || !h_witness || !r || !s || !proof256) return ZK_ERR_INVALID;
    if (comm->c->nranks == 1) return zk_groth16_prove(pk, r1cs, nullptr, h_witness, r, s, proof256, points);
    // A watchdog aborts this rank's communicator when the proof outlives
    // ZKML_SPLIT_TIMEOUT_S seconds (default 300): a rank whose peer died then
    // returns an error instead of waiting in a collective for good.
    const char* tv = getenv("ZKML_SPLIT_TIMEOUT_S");
    const double limit = tv && atof(tv) > 0 ? atof(tv) : 300.0;
    std::mutex mu;
    std::condition_variable cv;
    bool done = false, fired = false;
    std::thread dog([&]() {
        std::unique_lock<std::mutex> lk(mu);
        if (!cv.wait_for(lk, std::chrono::duration<double>(limit), [&] { return done; })) {
            fired = true;
            comm->c->abort();
        }
    });
    int rc = split::prove_split(pk, r1cs->r, comm->c, h_witness, r, s, proof256, points);
    {
        std::lock_guard<std::mutex> lk(mu);
        done = true;
    }
    cv.notify_all();
    dog.join();
    if (fired && rc == ZK_OK) rc = ZK_ERR_CUDA;  // the communicator is gone: later proofs cannot use it
    if (fired) set_error("split prove: rank %d exceeded %.0f s; its communicator was aborted", comm->c->rank, limit);
    return rc;
}

extern "C" int zk_groth16_prove_multi(zk_groth16_pk* const* pks, const zk_r1cs* const* r1cs, zk_comm* const* comms, int nranks,
                                      const void* h_witness, const void* r, const void* s, void* proof256, void* points,
                                      double timeout_s, zk_split_stats* stats) {
    clear_error();
    if (!pks || !r1cs || !comms || nranks < 1 || nranks > 64 || !h_witness || !r || !s || !proof256) return ZK_ERR_INVALID;
    for (int i = 0; i < nranks; i++)
        if (!pks[i] || !r1cs[i] || !comms[i] || !comms[i]->c || comms[i]->c->rank != i || comms[i]->c->nranks != nranks) {
            set_error("prove_multi: rank %d has no key, circuit or matching communicator", i);
            return ZK_ERR_INVALID;
        }
    std::vector<int> rc((size_t)nranks, ZK_OK);
    std::vector<std::string> err((size_t)nranks);
    std::vector<std::vector<uint8_t>> proofs((size_t)nranks, std::vector<uint8_t>(256));
    std::vector<std::vector<uint64_t>> pts((size_t)nranks, std::vector<uint64_t>(32));
    std::mutex mu;
    std::condition_variable cv;
    int finished = 0;
    std::vector<std::thread> th;
    for (int i = 0; i < nranks; i++) {
        th.emplace_back([&, i]() {
            int code = cudaSetDevice(comms[i]->c->device) == cudaSuccess ? ZK_OK : ZK_ERR_CUDA;
            if (code == ZK_OK)
                code = zk_groth16_prove_split(pks[i], r1cs[i], comms[i], h_witness, r, s, proofs[(size_t)i].data(),
                                              pts[(size_t)i].data());
            if (code != ZK_OK) {
                err[(size_t)i] = zk_last_error();
                for (int j = 0; j < nranks; j++) comms[j]->c->abort();  // no rank waits for this one
            }
            if (stats) zk_groth16_split_last_stats(&stats[i]);
            std::lock_guard<std::mutex> lk(mu);
            rc[(size_t)i] = code;
            finished++;
            cv.notify_all();
        });
    }
    {
        std::unique_lock<std::mutex> lk(mu);
        const bool all = cv.wait_for(lk, std::chrono::duration<double>(timeout_s > 0 ? timeout_s : 600.0),
                                     [&] { return finished == nranks; });
        if (!all) {
            lk.unlock();
            for (int j = 0; j < nranks; j++) comms[j]->c->abort();  // ends the waits of the ranks still running
        }
    }
    for (auto& t : th) t.join();
    for (int i = 0; i < nranks; i++)
        if (rc[(size_t)i] != ZK_OK) {
            set_error("prove_multi: rank %d: %s", i, err[(size_t)i].c_str());
            return rc[(size_t)i];
        }
    for (int i = 1; i < nranks; i++)
        if (proofs[(size_t)i] != proofs[0]) {
            set_error("prove_multi: ranks 0 and %d assembled different proofs", i);
            return ZK_ERR_CUDA;
        }
    std::memcpy(proof256, proofs[0].data(), 256);
    if (points) std::memcpy(points, pts[0].data(), 256);
    return ZK_OK;
}

extern "C" int zk_groth16_split_last_stats(zk_split_stats* out) {
    if (!out) return ZK_ERR_INVALID;
    *out = split::g_stats;
    return ZK_OK;
}
