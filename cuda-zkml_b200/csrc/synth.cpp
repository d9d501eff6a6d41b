// synth.cpp -- seeded synthetic R1CS workloads shaped like the reference's
// quantised-CNN statements (SURVEY configs 4/5): CONV2D 3x3 layers (pad 1)
// whose outputs go through an exact ReLU with a bit-decomposed range check and
// a right shift, then a dense layer.  The circuit comes with a satisfying
// witness, in the reference's data layout: constraints as
// zkml::SparseEntry records {int row; int col; Fr value} (40 bytes,
// src/prover/circuit.cuh:31-35) and the witness as Fr[num_variables] laid out
// [1, public..., private...] (src/prover/circuit.cuh:22-24).
//
// Constraint families (all coefficients small integers, converted to Montgomery
// form):
//   dot      sum_k W_k x_k + bias            * 1 = acc
//   bit      t_i                             * (t_i - 1) = 0        (b rows)
//   recomp   sum_i 2^i t_i - 2^(b-1)         * 1 = acc
//   relu     t_(b-1)                         * sum_{i=s}^{b-2} 2^(i-s) t_i = q
//   range    bits of q (o rows) and their recomposition
//   dense    sum_j V_kj q_j                  * 1 = out_k   (public outputs)
// The input feature map and the dense outputs are the public inputs.
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

int bitlen(uint64_t x) {
    int b = 0;
    while (x) { b++; x >>= 1; }
    return b;
}

}  // namespace

extern "C" int zk_synth_conv_circuit(int layers, int channels, int height, int width, int bits, int shift, int out_bits,
                                     int dense_outputs, uint64_t seed, zk_synth_circuit* out) {
    if (!out || layers < 1 || channels < 1 || height < 1 || width < 1 || bits < 4 || shift < 0 || out_bits < 0 ||
        dense_outputs < 0)
        return ZK_ERR_INVALID;
    std::memset(out, 0, sizeof *out);
    std::mt19937_64 rng(seed);
    auto i8 = [&]() { return (int64_t)(rng() % 255) - 127; };
    Builder B;
    const int C = channels, H = height, Wd = width, fm = C * H * Wd;
    const int num_public = fm + dense_outputs;
    B.wit.assign((size_t)1 + num_public, 0);
    B.wit[0] = 1;
    std::vector<int> X(fm);
    for (int i = 0; i < fm; i++) {
        X[i] = 1 + i;
        B.wit[(size_t)X[i]] = (int64_t)(rng() % 17);  // inputs in [0, 16]
    }
    for (int l = 0; l < layers; l++) {
        std::vector<int64_t> Wt((size_t)C * C * 9), bias(C);
        for (auto& w : Wt) w = i8();
        for (auto& b : bias) b = i8();
        // accumulators first, to size the range check of this layer
        std::vector<int64_t> acc(fm);
        int64_t amax = 0;
        for (int co = 0; co < C; co++)
            for (int y = 0; y < H; y++)
                for (int x = 0; x < Wd; x++) {
                    int64_t a = bias[co];
                    for (int ci = 0; ci < C; ci++)
                        for (int dy = 0; dy < 3; dy++)
                            for (int dx = 0; dx < 3; dx++) {
                                int yy = y + dy - 1, xx = x + dx - 1;
                                if (yy < 0 || yy >= H || xx < 0 || xx >= Wd) continue;
                                a += Wt[((size_t)co * C + ci) * 9 + dy * 3 + dx] * B.wit[(size_t)X[((size_t)ci * H + yy) * Wd + xx]];
                            }
                    acc[((size_t)co * H + y) * Wd + x] = a;
                    amax = std::max<int64_t>(amax, a < 0 ? -a : a);
                }
        const int b = std::max(bits, bitlen((uint64_t)amax) + 2);
        std::vector<int> Y(fm);
        for (int co = 0; co < C; co++)
            for (int y = 0; y < H; y++)
                for (int x = 0; x < Wd; x++) {
                    const size_t o = ((size_t)co * H + y) * Wd + x;
                    const int64_t a = acc[o];
                    const int av = B.var(a);
                    // dot: sum W x + bias = acc
                    int row = B.rows++;
                    for (int ci = 0; ci < C; ci++)
                        for (int dy = 0; dy < 3; dy++)
                            for (int dx = 0; dx < 3; dx++) {
                                int yy = y + dy - 1, xx = x + dx - 1;
                                if (yy < 0 || yy >= H || xx < 0 || xx >= Wd) continue;
                                B.put(0, row, X[((size_t)ci * H + yy) * Wd + xx], Wt[((size_t)co * C + ci) * 9 + dy * 3 + dx]);
                            }
                    B.put(0, row, 0, bias[co]);
                    B.put(1, row, 0, 1);
                    B.put(2, row, av, 1);
                    // bit decomposition of t = acc + 2^(b-1)
                    const uint64_t t = (uint64_t)(a + ((int64_t)1 << (b - 1)));
                    std::vector<int> tv(b);
                    for (int i = 0; i < b; i++) {
                        tv[i] = B.var((int64_t)((t >> i) & 1));
                        row = B.rows++;
                        B.put(0, row, tv[i], 1);
                        B.put(1, row, tv[i], 1);
                        B.put(1, row, 0, -1);
                    }
                    row = B.rows++;
                    for (int i = 0; i < b; i++) B.put(0, row, tv[i], (int64_t)1 << i);
                    B.put(0, row, 0, -((int64_t)1 << (b - 1)));
                    B.put(1, row, 0, 1);
                    B.put(2, row, av, 1);
                    // relu + shift: q = sign * floor(t_low / 2^s)
                    const int64_t q = a > 0 ? (a >> shift) : 0;
                    const int qv = B.var(q);
                    row = B.rows++;
                    B.put(0, row, tv[b - 1], 1);
                    for (int i = shift; i <= b - 2; i++) B.put(1, row, tv[i], (int64_t)1 << (i - shift));
                    B.put(2, row, qv, 1);
                    // range check of q (at least as many bits as q can have)
                    const int ob = out_bits > 0 ? std::max(out_bits, b - 1 - shift) : 0;
                    if (ob > 0) {
                        std::vector<int> uv(ob);
                        for (int i = 0; i < ob; i++) {
                            uv[i] = B.var((int64_t)(((uint64_t)q >> i) & 1));
                            row = B.rows++;
                            B.put(0, row, uv[i], 1);
                            B.put(1, row, uv[i], 1);
                            B.put(1, row, 0, -1);
                        }
                        row = B.rows++;
                        for (int i = 0; i < ob; i++) B.put(0, row, uv[i], (int64_t)1 << i);
                        B.put(1, row, 0, 1);
                        B.put(2, row, qv, 1);
                    }
                    Y[o] = qv;
                }
        X.swap(Y);
    }
    for (int k = 0; k < dense_outputs; k++) {
        const int ov = 1 + fm + k;
        int64_t s = 0;
        const int row = B.rows++;
        for (int j = 0; j < fm; j++) {
            const int64_t v = i8();
            if (!v) continue;
            B.put(0, row, X[j], v);
            s += v * B.wit[(size_t)X[j]];
        }
        B.put(1, row, 0, 1);
        B.put(2, row, ov, 1);
        B.wit[(size_t)ov] = s;
    }
    const size_t m = B.wit.size();
    zkh::Fe* w = (zkh::Fe*)std::malloc(m * 32);
    if (!w) return ZK_ERR_NOMEM;
    for (size_t i = 0; i < m; i++) w[i] = B.fr_of(B.wit[i]);
    for (int k = 0; k < 3; k++) {
        out->nnz[k] = B.m[k].size();
        out->entries[k] = std::malloc(std::max<size_t>(1, B.m[k].size()) * sizeof(Entry));
        if (!out->entries[k]) return ZK_ERR_NOMEM;
        std::memcpy(out->entries[k], B.m[k].data(), B.m[k].size() * sizeof(Entry));
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
