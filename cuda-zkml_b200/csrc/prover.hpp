// prover.hpp -- the device-resident constraint system and proving key shared
// by the one-device prover (groth16.cu) and the prover split over several
// devices (split.cu), with the pieces of a prove both use.
#pragma once
#include "field.cuh"
#include "host_field.hpp"
#include "runtime.cuh"

#include <map>
#include <mutex>
#include <utility>
#include <vector>

namespace zk {

// ------------------------------------------------------------------ R1CS
struct SparseEntry {  // zkml::SparseEntry (src/prover/circuit.cuh:31-35)
    int32_t row;
    int32_t col;
    uint64_t v[4];
};
static_assert(sizeof(SparseEntry) == 40, "SparseEntry layout");

struct Csr {
    std::vector<int32_t> row_ptr, col;
    std::vector<zkh::Fe> val;
    std::vector<int32_t> mid_rows;   // rows with kShortRow < entries <= kMidRow (ascending)
    std::vector<int32_t> long_rows;  // rows with > kMidRow entries (ascending)
};
// Row lengths: up to kShortRow entries one thread per row, up to kMidRow one
// warp per row (the 289-entry rows of a 3x3x32 convolution), beyond that one
// block per row (dense layers).  A block per 289-entry row left most of its
// threads idle through a synchronised shared-memory tree.
static constexpr int kShortRow = 16;
static constexpr int kMidRow = 2048;

struct R1cs {
    int device = -1;
    int num_constraints = 0, m = 0, num_public = 0, log_n = 0;
    uint64_t n = 0;
    Csr host[3];
    int32_t* d_row_ptr[3] = {};
    int32_t* d_col[3] = {};
    Fr* d_val[3] = {};
    int32_t* d_mid[3] = {};
    int32_t* d_long[3] = {};
    size_t nnz[3] = {};
};

namespace split { struct State; }

}  // namespace zk

struct zk_r1cs {
    zk::R1cs r;
};

struct zk_groth16_pk {
    int device = -1;
    int num_constraints = 0;  // padded domain size n, as the reference stores it (groth16.cu:621)
    int m = 0, num_public = 0, l = 0, n_h = 0;
    uint8_t* g1 = nullptr;  // device: A[m] | B1[m] | L[l] | H[n_h]   (64-B packed)
    uint8_t* g2 = nullptr;  // device: B2[m]                          (128-B packed)
    uint64_t alpha1[8], beta1[8], delta1[8];
    uint64_t beta2[16], gamma2[16], delta2[16], g2gen[16], tau2[16];
    std::vector<uint64_t> ic;  // (num_public + 1) x 8
    // prover buffers
    zk::Fr* w = nullptr;
    zk::Fr* abc = nullptr;  // 3 n
    zk::Fr* h = nullptr;    // n
    unsigned long long* d_bad = nullptr;  // first failing constraint of the witness check
    unsigned long long* h_bad = nullptr;  // pinned host copy
    uint64_t n_buf = 0;
    // 2^i delta1 and 2^i delta2 (i < 256), built on first use: r delta1 and
    // s delta2 of every proof as sums of table entries
    mutable std::mutex tab_mu;
    mutable std::vector<zkh::Xyzz<zkh::Fe>> d1_pow;
    mutable std::vector<zkh::Xyzz<zkh::Fp2>> d2_pow;
    // window tables of the H query (2^(c j) H_i, j < h_W).  The first proof
    // that finds none starts their build on a stream of its own and runs its H
    // MSM without them; a later call publishes them once the build's event has
    // fired (zk_groth16_precompute builds them and waits).
    uint8_t* h_tab = nullptr;
    int h_c = 0, h_W = 0;
    uint8_t* h_tab_pending = nullptr;
    int h_pc = 0, h_pW = 0;
    bool h_tab_off = false;  // no device memory for them: proofs keep the plain MSM
    cudaStream_t h_tab_stream = nullptr;
    cudaEvent_t h_tab_done = nullptr;
    std::mutex h_mu;
    // private device context of the witness MSMs inside prove (created on first
    // use), so that they run beside compute_h and the H MSM on the shared one
    zk::DeviceContext* wctx = nullptr;
    // the one-device proof's critical path runs on this highest-priority stream
    cudaStream_t prio_stream = nullptr;
    // per (log_parts, part): that part's H points in the "blocks" order of a
    // proof split over 2^log_parts parts, and window tables over them; built on
    // first use and kept until the key is destroyed (a process proving one part
    // holds one entry; ranks emulated as threads on one device hold several)
    struct HBlocks {
        uint8_t* pts = nullptr;
        uint8_t* tab = nullptr;
        int c = 0, W = 0;
    };
    std::map<std::pair<int, int>, HBlocks> hb;
    // per (ranks, rank): buffers of a prove split over that many ranks (split.cu)
    std::map<std::pair<int, int>, zk::split::State*> split;
};

namespace zk {

// rows [lo, hi) of A w, B w, C w into out3 (three vectors of hi - lo elements);
// rows at or beyond the constraint count are zero
int r1cs_matvec_rows(const R1cs& R, cudaStream_t st, const Fr* w, uint64_t lo, uint64_t hi, Fr* out3, int num_sms);
// the reference's verify_witness on rows [row0, row0 + count): *first_bad
// (device, starting at 0xff..ff) ends as the first failing row, if any
void enqueue_hadamard_check(cudaStream_t st, const Fr* a, const Fr* b, const Fr* c, uint64_t count, uint64_t row0,
                            unsigned long long* first_bad, int num_sms);
// false when ZKML_SKIP_WITNESS_CHECK=1
bool witness_check_enabled();
// the key's private device context of the witness MSMs (created on first use)
int ensure_witness_context(zk_groth16_pk* pk);
// A, B2, B1 and L over the witness slice [lo, hi) (one shared sort) in `ctx`
int witness_msms(zk_groth16_pk* pk, DeviceContext* ctx, cudaStream_t st, const Fr* d_w, size_t lo, size_t hi, uint64_t a[8],
                 uint64_t b[16], uint64_t b1[8], uint64_t l[8], float set_ms[4], float* all_ms);
// one part's share of the H MSM in the "blocks" layout of a split transform
int h_msm_blocks(zk_groth16_pk* pk, cudaStream_t st, const Fr* d_h_part, int log_parts, int part, uint64_t out[8]);
// frees the split-prove buffers held by a key (split.cu)
void destroy_split_states(zk_groth16_pk* pk);

}  // namespace zk
