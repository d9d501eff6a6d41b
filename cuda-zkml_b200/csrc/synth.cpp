// synth.cpp -- seeded synthetic R1CS workloads with the constraint structure
// of the reference's quantised-CNN statements (statement v2 with fixed model
// weights, src/prover/statement_v2.cuh:98-240, gadgets from
// src/prover/gadgets.cuh): CONV2D 3x3 layers (pad 1) whose outputs go through
// RELU_EXACT (an exact ReLU plus a range-checked rescale), then a dense layer
// whose outputs are public.  The circuit comes with a satisfying witness, in the
// reference's data layout: constraints as zkml::SparseEntry records
// {int row; int col; Fr value} (40 bytes, src/prover/circuit.cuh:31-35) and the
// witness as Fr[num_variables] laid out [1, public..., private...]
// (src/prover/circuit.cuh:22-24).
//
// Variables, in allocation order (statement_v2.cuh:111-128): the constant 1,
// the public dense outputs, the public model tag, the public input feature
// map; then per layer the conv outputs, then per neuron the ReLU and rescale
// variables; last the dense outputs' private copies.  Rows, in order, with
// k the layer's range width and s the shift:
//   tag       tag * 1 = tag_var                                 (1 row)
//   conv      sum_taps W x + bias * 1 = z    (add_fixed_conv2d, gadgets.cuh:281-311;
//             taps with a zero weight are skipped, the bias term is always kept)
//   ReLU      b_i * (b_i - 1) = 0, i < k; sum 2^i b_i - z - 2^(k-1) = 0;
//             b_(k-1) * z = y                 (add_relu_exact, gadgets.cuh:197-204)
//   rescale   bits of r (s rows + recomposition), signed bits of q (k rows +
//             recomposition), q 2^s + r - y = 0   (add_rescale, gadgets.cuh:207-220)
//   dense     sum_j V_kj q_j + bias * 1 = out_k             (add_fixed_linear)
//   outputs   pub_k - out_k = 0                        (statement_v2.cuh:216-218)
// A config-5 shape (2 layers of 32 x 32 x 32, k = 24 then 23, s = 10, 10 dense
// outputs) gives 4,128,789 constraints and 4,030,486 variables (32,779 public),
// the counts of the reference's own statement for that model.
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <random>
#include <vector>

#include "../../include/zkml_b200.h"
#include "host_field.hpp"

namespace {

struct Entry {  // zkml::SparseEntry layout
    int32_t row;
    int32_t col;
    uint64_t v[4];
};
static_assert(sizeof(Entry) == 40, "SparseEntry layout");

struct Builder {
    std::vector<Entry> m[3];
    std::vector<int64_t> wit;  // small-integer witness values (exact)
    int rows = 0;
    std::vector<zkh::Fe> small_cache;  // Montgomery forms of -1024..1024

    zkh::Fe fr_of(int64_t v) {
        if (v >= -1024 && v <= 1024) return small_cache[(size_t)(v + 1024)];
        uint64_t s[4] = {(uint64_t)(v < 0 ? -v : v), 0, 0, 0};
        zkh::Fe f;
        zkh::from_std(zkh::kR, f, s);
        if (v < 0) zkh::sub(zkh::kR, f, zkh::zero(), f);
        return f;
    }
    Builder() {
        small_cache.resize(2049);
        for (int64_t v = -1024; v <= 1024; v++) {
            uint64_t s[4] = {(uint64_t)(v < 0 ? -v : v), 0, 0, 0};
            zkh::Fe f;
            zkh::from_std(zkh::kR, f, s);
            if (v < 0) zkh::sub(zkh::kR, f, zkh::zero(), f);
            small_cache[(size_t)(v + 1024)] = f;
        }
    }
    void put(int which, int row, int col, int64_t coeff) {
        Entry e;
        e.row = row;
        e.col = col;
        zkh::Fe f = fr_of(coeff);
        std::memcpy(e.v, f.v, 32);
        m[which].push_back(e);
    }
    int var(int64_t value) {
        wit.push_back(value);
        return (int)wit.size() - 1;
    }
};


}  // namespace

extern "C" int zk_synth_conv_circuit(int layers, int channels, int height, int width, int bits, int shift, int out_bits,
                                     int dense_outputs, uint64_t seed, zk_synth_circuit* out) {
    if (!out || layers < 1 || channels < 1 || height < 1 || width < 1 || bits < 2 || bits > 60 || shift < 0 ||
        shift > 60 || out_bits < 0 || out_bits == 1 || out_bits > 60 || dense_outputs < 0)
        return ZK_ERR_INVALID;
    std::memset(out, 0, sizeof *out);
    std::mt19937_64 rng(seed);
    auto i8 = [&]() { return (int64_t)(rng() % 255) - 127; };
    Builder B;
    const int C = channels, H = height, Wd = width, fm = C * H * Wd;
    // public: [dense outputs, model tag, input feature map]
    const int num_public = dense_outputs + 1 + fm;
    B.wit.assign((size_t)1 + num_public, 0);
    B.wit[0] = 1;
    const int tag = 1 + dense_outputs;
    const int64_t tag_value = (int64_t)(rng() >> 2);
    B.wit[(size_t)tag] = tag_value;
    std::vector<int> X(fm);
    for (int i = 0; i < fm; i++) {
        X[i] = tag + 1 + i;
        B.wit[(size_t)X[i]] = (int64_t)(rng() % 17);  // inputs in [0, 16]
    }
    int row = B.rows++;
    B.put(0, row, 0, tag_value);
    B.put(1, row, 0, 1);
    B.put(2, row, tag, 1);

    // k boolean variables for v + offset (LSB first), their b (b - 1) = 0 rows and
    // the recomposition row sum 2^i b_i - v - offset = 0 (no offset term when 0)
    auto range_bits = [&](int v, int64_t offset, int k) -> int {
        const uint64_t t = (uint64_t)(B.wit[(size_t)v] + offset);
        int first = -1;
        for (int i = 0; i < k; i++) {
            const int bv = B.var((int64_t)((t >> i) & 1));
            if (i == 0) first = bv;
            const int r = B.rows++;
            B.put(0, r, bv, 1);
            B.put(1, r, bv, 1);
            B.put(1, r, 0, -1);
        }
        const int r = B.rows++;
        for (int i = 0; i < k; i++) B.put(0, r, first + i, (int64_t)1 << i);
        B.put(0, r, v, -1);
        if (offset) B.put(0, r, 0, -offset);
        B.put(1, r, 0, 1);
        return first;
    };

    for (int l = 0; l < layers; l++) {
        const int k = (l == 0 || out_bits == 0) ? bits : out_bits;
        const int64_t half = (int64_t)1 << (k - 1);
        std::vector<int64_t> Wt((size_t)C * C * 9), bias(C);
        for (auto& w : Wt) w = i8();
        for (auto& b : bias) b = i8();
        std::vector<int> Z(fm);
        for (int co = 0; co < C; co++)
            for (int y = 0; y < H; y++)
                for (int x = 0; x < Wd; x++) {
                    const size_t o = ((size_t)co * H + y) * Wd + x;
                    row = B.rows++;
                    int64_t a = bias[co];
                    for (int ci = 0; ci < C; ci++)
                        for (int dy = 0; dy < 3; dy++)
                            for (int dx = 0; dx < 3; dx++) {
                                const int yy = y + dy - 1, xx = x + dx - 1;
                                if (yy < 0 || yy >= H || xx < 0 || xx >= Wd) continue;
                                const int64_t w = Wt[((size_t)co * C + ci) * 9 + dy * 3 + dx];
                                if (!w) continue;
                                const int xv = X[((size_t)ci * H + yy) * Wd + xx];
                                B.put(0, row, xv, w);
                                a += w * B.wit[(size_t)xv];
                            }
                    B.put(0, row, 0, bias[co]);
                    B.put(1, row, 0, 1);
                    Z[o] = B.var(a);
                    B.put(2, row, Z[o], 1);
                    if (a < -half || a >= half) return ZK_ERR_INVALID;  // outside the layer's range
                }
        std::vector<int> Q(fm);
        for (size_t o = 0; o < (size_t)fm; o++) {
            const int z = Z[o];
            const int64_t a = B.wit[(size_t)z];
            // exact ReLU: the top bit of z + 2^(k-1) is [z >= 0]; y = s z
            const int b0 = range_bits(z, half, k);
            const int s = b0 + k - 1;
            const int yv = B.var(B.wit[(size_t)s] * a);
            row = B.rows++;
            B.put(0, row, s, 1);
            B.put(1, row, z, 1);
            B.put(2, row, yv, 1);
            if (shift == 0) {
                Q[o] = yv;
                continue;
            }
            // rescale: y = q 2^s + r with 0 <= r < 2^s and q in the signed k-bit range
            const int64_t y = B.wit[(size_t)yv];
            const int64_t q = y >> shift, r = y - (q << shift);
            if (q < -half || q >= half) return ZK_ERR_INVALID;
            const int qv = B.var(q), rv = B.var(r);
            range_bits(rv, 0, shift);
            range_bits(qv, half, k);
            row = B.rows++;
            B.put(0, row, qv, (int64_t)1 << shift);
            B.put(0, row, rv, 1);
            B.put(0, row, yv, -1);
            B.put(1, row, 0, 1);
            Q[o] = qv;
        }
        X.swap(Q);
    }
    std::vector<int> dense(dense_outputs);
    for (int kk = 0; kk < dense_outputs; kk++) {
        row = B.rows++;
        int64_t s = 0;
        for (int j = 0; j < fm; j++) {
            const int64_t v = i8();
            if (!v) continue;
            B.put(0, row, X[j], v);
            s += v * B.wit[(size_t)X[j]];
        }
        const int64_t b = i8();
        B.put(0, row, 0, b);
        s += b;
        B.put(1, row, 0, 1);
        dense[kk] = B.var(s);
        B.put(2, row, dense[kk], 1);
    }
    for (int kk = 0; kk < dense_outputs; kk++) {
        const int pv = 1 + kk;
        B.wit[(size_t)pv] = B.wit[(size_t)dense[kk]];
        row = B.rows++;
        B.put(0, row, pv, 1);
        B.put(0, row, dense[kk], -1);
        B.put(1, row, 0, 1);
    }
    const size_t m = B.wit.size();
    zkh::Fe* w = (zkh::Fe*)std::malloc(m * 32);
    if (!w) return ZK_ERR_NOMEM;
    for (size_t i = 0; i < m; i++) w[i] = B.fr_of(B.wit[i]);
    for (int kk = 0; kk < 3; kk++) {
        out->nnz[kk] = B.m[kk].size();
        out->entries[kk] = std::malloc(std::max<size_t>(1, B.m[kk].size()) * sizeof(Entry));
        if (!out->entries[kk]) {
            std::free(w);
            zk_synth_free(out);
            return ZK_ERR_NOMEM;
        }
        std::memcpy(out->entries[kk], B.m[kk].data(), B.m[kk].size() * sizeof(Entry));
    }
    out->witness = w;
    out->num_constraints = B.rows;
    out->num_variables = (int)m;
    out->num_public = num_public;
    return ZK_OK;
}

// A quantised MLP statement (statement v2 with fixed weights and a context
// binding, src/prover/statement_v2.cuh:98-240): `batch` samples of
// n_in -> n_hidden (LINEAR, then RELU_EXACT with `bits` and `shift`) -> n_out
// (LINEAR), one seeded int8 model for all samples, inputs in 0..16.  Public, in
// order: the batch x n_out outputs, the model tag, the context (when `context`),
// the batch x n_in inputs.  Rows: the tag, the context binding ctx * ctx = ctx^2
// (add_context_binding, gadgets.cuh:152-158), then per sample the linear rows,
// each hidden neuron's ReLU and rescale rows, the output rows and the
// output-equality rows.  Batch 4 of 64 -> 32 -> 10 with bits 24, shift 6 gives
// 7,762 constraints, 7,764 variables and 298 public, the counts of the
// reference's own statement for that model.
extern "C" int zk_synth_mlp_circuit(int batch, int n_in, int n_hidden, int n_out, int bits, int shift, int context, uint64_t seed,
                                    zk_synth_circuit* out) {
    if (!out || batch < 1 || n_in < 1 || n_hidden < 1 || n_out < 1 || bits < 2 || bits > 60 || shift < 0 || shift > 60)
        return ZK_ERR_INVALID;
    std::memset(out, 0, sizeof *out);
    std::mt19937_64 rng(seed);
    auto i8 = [&]() { return (int64_t)(rng() % 255) - 127; };
    std::vector<int64_t> W1((size_t)n_hidden * n_in), b1(n_hidden), W2((size_t)n_out * n_hidden), b2(n_out);
    for (auto& w : W1) w = i8();
    for (auto& b : b1) b = i8();
    for (auto& w : W2) w = i8();
    for (auto& b : b2) b = i8();
    Builder B;
    const int outs = 1, tag = outs + batch * n_out, ctx = tag + 1, ins = ctx + (context ? 1 : 0);
    const int num_public = batch * n_out + 1 + (context ? 1 : 0) + batch * n_in;
    B.wit.assign((size_t)1 + num_public, 0);
    B.wit[0] = 1;
    const int64_t tag_value = (int64_t)(rng() >> 2);
    B.wit[(size_t)tag] = tag_value;
    int row = B.rows++;
    B.put(0, row, 0, tag_value);
    B.put(1, row, 0, 1);
    B.put(2, row, tag, 1);
    if (context) {
        const int64_t c = (int64_t)(rng() >> 33);  // c^2 stays an exact int64
        B.wit[(size_t)ctx] = c;
        const int sq = B.var(c * c);
        row = B.rows++;
        B.put(0, row, ctx, 1);
        B.put(1, row, ctx, 1);
        B.put(2, row, sq, 1);
    }
    for (int i = 0; i < batch * n_in; i++) B.wit[(size_t)(ins + i)] = (int64_t)(rng() % 17);
    const int64_t half = (int64_t)1 << (bits - 1);
    auto range_bits = [&](int v, int64_t offset, int k) -> int {
        const uint64_t t = (uint64_t)(B.wit[(size_t)v] + offset);
        int first = -1;
        for (int i = 0; i < k; i++) {
            const int bv = B.var((int64_t)((t >> i) & 1));
            if (i == 0) first = bv;
            const int r = B.rows++;
            B.put(0, r, bv, 1);
            B.put(1, r, bv, 1);
            B.put(1, r, 0, -1);
        }
        const int r = B.rows++;
        for (int i = 0; i < k; i++) B.put(0, r, first + i, (int64_t)1 << i);
        B.put(0, r, v, -1);
        if (offset) B.put(0, r, 0, -offset);
        B.put(1, r, 0, 1);
        return first;
    };
    // y = W x + b, one row per output (add_fixed_linear; zero weights skipped, the bias kept)
    auto linear = [&](const std::vector<int>& x, const std::vector<int64_t>& W, const std::vector<int64_t>& bias, int n_o) {
        std::vector<int> y(n_o);
        for (int o = 0; o < n_o; o++) {
            const int r = B.rows++;
            int64_t acc = bias[o];
            for (size_t j = 0; j < x.size(); j++) {
                const int64_t w = W[(size_t)o * x.size() + j];
                if (!w) continue;
                B.put(0, r, x[j], w);
                acc += w * B.wit[(size_t)x[j]];
            }
            B.put(0, r, 0, bias[o]);
            B.put(1, r, 0, 1);
            y[o] = B.var(acc);
            B.put(2, r, y[o], 1);
        }
        return y;
    };
    for (int b = 0; b < batch; b++) {
        std::vector<int> x(n_in);
        for (int i = 0; i < n_in; i++) x[i] = ins + b * n_in + i;
        std::vector<int> h = linear(x, W1, b1, n_hidden);
        for (auto& z : h) {
            const int64_t a = B.wit[(size_t)z];
            if (a < -half || a >= half) return ZK_ERR_INVALID;  // outside the ReLU's range
            const int s = range_bits(z, half, bits) + bits - 1;
            const int yv = B.var(B.wit[(size_t)s] * a);
            row = B.rows++;
            B.put(0, row, s, 1);
            B.put(1, row, z, 1);
            B.put(2, row, yv, 1);
            if (shift == 0) {
                z = yv;
                continue;
            }
            const int64_t y = B.wit[(size_t)yv];
            const int64_t q = y >> shift, r = y - (q << shift);
            if (q < -half || q >= half) return ZK_ERR_INVALID;
            const int qv = B.var(q), rv = B.var(r);
            range_bits(rv, 0, shift);
            range_bits(qv, half, bits);
            row = B.rows++;
            B.put(0, row, qv, (int64_t)1 << shift);
            B.put(0, row, rv, 1);
            B.put(0, row, yv, -1);
            B.put(1, row, 0, 1);
            z = qv;
        }
        std::vector<int> y = linear(h, W2, b2, n_out);
        for (int o = 0; o < n_out; o++) {
            const int pv = outs + b * n_out + o;
            B.wit[(size_t)pv] = B.wit[(size_t)y[o]];
            row = B.rows++;
            B.put(0, row, pv, 1);
            B.put(0, row, y[o], -1);
            B.put(1, row, 0, 1);
        }
    }
    const size_t m = B.wit.size();
    zkh::Fe* w = (zkh::Fe*)std::malloc(m * 32);
    if (!w) return ZK_ERR_NOMEM;
    for (size_t i = 0; i < m; i++) w[i] = B.fr_of(B.wit[i]);
    for (int kk = 0; kk < 3; kk++) {
        out->nnz[kk] = B.m[kk].size();
        out->entries[kk] = std::malloc(std::max<size_t>(1, B.m[kk].size()) * sizeof(Entry));
        if (!out->entries[kk]) {
            std::free(w);
            zk_synth_free(out);
            return ZK_ERR_NOMEM;
        }
        std::memcpy(out->entries[kk], B.m[kk].data(), B.m[kk].size() * sizeof(Entry));
    }
    out->witness = w;
    out->num_constraints = B.rows;
    out->num_variables = (int)m;
    out->num_public = num_public;
    return ZK_OK;
}

extern "C" void zk_synth_free(zk_synth_circuit* c) {
    if (!c) return;
    for (int k = 0; k < 3; k++) std::free(c->entries[k]);
    std::free(c->witness);
    std::memset(c, 0, sizeof *c);
}
