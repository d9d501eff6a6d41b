// ref_statement_driver.cpp -- builds R1CS + witness with the reference's own
// statement-v2 builder (build_statement_v2, src/prover/statement_v2.cuh:82-257,
// over the gadgets of src/prover/gadgets.cuh), for the Groth16 parity tests.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile with g++ from the
// reference's headers where they lie, through the reference's own host shim
// (tests/host/shim/cuda_runtime.h), into oracle/_ref/libzkref_stmt.so.  Nothing
// in the library under test links or loads it.
//
// Statements:
//   * ref_stmt_mlp: a quantised MLP n_in -> n_hidden (LINEAR + RELU_EXACT) ->
//     n_out (LINEAR) with given integer weights, public inputs and outputs,
//     a model tag and an optional context binding (the "context-bound public
//     statement" of the zkml-prove CLI's --statement-v2, src/cli/prove.cu:
//     1168-1201).  Batch 4 of 64 -> 32 (bits 24, shift 6) -> 10 gives 7,762
//     constraints.
//   * ref_stmt_tiny_cnn: the reference host test's tiny CNN and batch of two
//     (tests/host/test_statement_v2.cpp:28-43, :99-105) with its variant A
//     (public model, inputs and outputs, context-bound; 8,082 constraints) or
//     variant B (Poseidon-committed private model, committed private inputs,
//     private outputs, in-circuit routing; 62,692 constraints), options as in
//     that test (:107-139).
#include "prover/statement_v2.cuh"

#include <cstdlib>
#include <cstring>

using namespace zkml;
using bn254::Fp;

extern "C" {

typedef struct {
    int num_constraints, num_variables, num_public;
    size_t nnz[3];
    void* entries[3];  // SparseEntry {int32 row; int32 col; Fr value} (40 B)
    void* witness;     // Fr[num_variables], Montgomery
} ref_circuit;

void ref_circuit_free(ref_circuit* c) {
    if (!c) return;
    for (int k = 0; k < 3; k++) free(c->entries[k]);
    free(c->witness);
    std::memset(c, 0, sizeof *c);
}

}  // extern "C"

static int export_statement(const StatementV2& st, ref_circuit* out) {
    static_assert(sizeof(SparseEntry) == 40, "SparseEntry layout");
    std::memset(out, 0, sizeof *out);
    const R1CS& r = st.r1cs;
    out->num_constraints = r.num_constraints;
    out->num_variables = r.num_variables;
    out->num_public = st.layout.num_public;
    const std::vector<SparseEntry>* mats[3] = {&r.A, &r.B, &r.C};
    for (int k = 0; k < 3; k++) {
        out->nnz[k] = mats[k]->size();
        out->entries[k] = malloc(std::max<size_t>(1, mats[k]->size()) * sizeof(SparseEntry));
        std::memcpy(out->entries[k], mats[k]->data(), mats[k]->size() * sizeof(SparseEntry));
    }
    out->witness = malloc(st.witness.values.size() * sizeof(bn254::Fr));
    std::memcpy(out->witness, st.witness.values.data(), st.witness.values.size() * sizeof(bn254::Fr));
    if (st.witness.num_public != st.layout.num_public || (int)st.witness.values.size() != r.num_variables) return 3;
    return r.verify_witness(st.witness.values) ? 0 : 4;
}

extern "C" {

// weights: w1[n_hidden * n_in], b1[n_hidden], w2[n_out * n_hidden], b2[n_out]
// (row-major, out x in); inputs[batch * n_in].  Returns 0, or 1 when the
// builder refuses (a value outside its range), 3/4 on an inconsistent or
// unsatisfied statement.
int ref_stmt_mlp(int batch, int n_in, int n_hidden, int n_out, int bits, int shift, int context, uint64_t model_tag,
                 const int32_t* w1, const int32_t* b1, const int32_t* w2, const int32_t* b2, const int32_t* inputs,
                 ref_circuit* out) {
    NNModel m;
    m.layers.push_back(NNModel::make_linear_layer(n_in, n_hidden));
    m.layers.push_back(NNModel::make_relu_exact_layer(n_hidden, bits, shift));
    m.layers.push_back(NNModel::make_linear_layer(n_hidden, n_out));
    m.layers.push_back(NNModel::make_softmax_layer(n_out));
    for (size_t i = 0; i < m.layers[0].weights.size(); i++) m.layers[0].weights[i] = i64_to_fp(w1[i]);
    for (size_t i = 0; i < m.layers[0].bias.size(); i++) m.layers[0].bias[i] = i64_to_fp(b1[i]);
    for (size_t i = 0; i < m.layers[2].weights.size(); i++) m.layers[2].weights[i] = i64_to_fp(w2[i]);
    for (size_t i = 0; i < m.layers[2].bias.size(); i++) m.layers[2].bias[i] = i64_to_fp(b2[i]);
    std::vector<std::vector<Fp>> xs((size_t)batch, std::vector<Fp>((size_t)n_in));
    for (int b = 0; b < batch; b++)
        for (int i = 0; i < n_in; i++) xs[(size_t)b][(size_t)i] = i64_to_fp(inputs[(size_t)b * n_in + i]);
    StatementV2Options o;
    o.model_tag = Fr::from_uint(model_tag);
    if (context) {
        o.has_context = true;
        fr_from_hex("0x0123456789abcdef0123456789abcdef", &o.context);  // tests/host/test_statement_v2.cpp:111
    }
    StatementV2 st;
    std::string err;
    if (!build_statement_v2(m, xs, o, st, err)) return 1;
    return export_statement(st, out);
}

// variant 0: A, 1: B of tests/host/test_statement_v2.cpp
int ref_stmt_tiny_cnn(int variant, ref_circuit* out) {
    NNModel m;
    Conv2DParams c;
    c.in_c = 1; c.in_h = 6; c.in_w = 6; c.out_c = 2; c.kh = 3; c.kw = 3; c.stride = 1; c.pad = 1;
    m.layers.push_back(NNModel::make_conv2d_layer(c));
    m.layers.push_back(NNModel::make_relu_exact_layer(c.out_size(), 24, 2));
    m.layers.push_back(NNModel::make_linear_layer(c.out_size(), 4));
    m.layers.push_back(NNModel::make_softmax_layer(4));
    auto& conv = m.layers[0];
    for (size_t i = 0; i < conv.weights.size(); i++) conv.weights[i] = i64_to_fp((int64_t)((i * 5) % 7) - 3);
    conv.bias[0] = i64_to_fp(4);
    conv.bias[1] = i64_to_fp(-2);
    auto& lin = m.layers[2];
    for (size_t i = 0; i < lin.weights.size(); i++) lin.weights[i] = i64_to_fp((int64_t)((i * 3) % 9) - 4);
    for (size_t i = 0; i < lin.bias.size(); i++) lin.bias[i] = i64_to_fp((int64_t)i - 1);
    std::vector<std::vector<Fp>> batch(2, std::vector<Fp>(36));
    for (int i = 0; i < 36; i++) {
        batch[0][(size_t)i] = i64_to_fp((i * 7) % 13 - 4);
        batch[1][(size_t)i] = i64_to_fp((i * 11) % 17 - 8);
    }
    StatementV2Options o;
    o.model_tag = Fr::from_uint(0xC0FFEE);
    if (variant == 0) {
        o.has_context = true;
        fr_from_hex("0x0123456789abcdef0123456789abcdef", &o.context);
    } else {
        o.private_input = true;
        o.input_blinding = {Fr::from_uint(0x5EED1), Fr::from_uint(0x5EED2)};
        o.private_model = true;
        o.private_outputs = true;
        o.route = true;
        o.route_threshold = 5;
    }
    StatementV2 st;
    std::string err;
    if (!build_statement_v2(m, batch, o, st, err)) return 1;
    return export_statement(st, out);
}

}  // extern "C"
