"""The seeded synthetic CONV/RELU_EXACT circuits (host code, no GPU): their
witnesses satisfy them, a changed witness value breaks the right rows, and the
config-5 shape has the constraint and variable counts of the reference's own
statement for that model (statement v2 with fixed weights: 2 x CONV2D 3x3
32->32 ch on 32 x 32 with RELU_EXACT bits 24 then 23, shift 10, then
LINEAR 32768 -> 10)."""
import numpy as np
import pytest

import groth16_oracle as G
import zkml_b200 as Z

SMALL = [
    (1, 2, 4, 4, 24, 10, 0, 2, 21),
    (2, 2, 4, 4, 24, 10, 23, 3, 7),
    (2, 3, 5, 6, 20, 8, 18, 4, 3),
    (1, 1, 3, 3, 24, 0, 0, 1, 5),  # shift 0: no rescale rows
]


def _rows_per_neuron(k, shift):
    # conv 1; ReLU k bits + recomposition + y = s z; rescale shift bits + recomposition,
    # k bits + recomposition, q 2^s + r = y  (src/prover/gadgets.cuh:197-220)
    return 1 + (k + 2) + ((shift + 1) + (k + 1) + 1 if shift else 0)


def _vars_per_neuron(k, shift):
    return 1 + (k + 1) + ((2 + shift + k) if shift else 0)


@pytest.mark.parametrize("args", SMALL)
def test_small_circuits_are_satisfied(args):
    layers, ch, h, w, bits, shift, out_bits, dense, seed = args
    c = Z.synth_conv_circuit(*args)
    fm = ch * h * w
    ks = [bits if (l == 0 or out_bits == 0) else out_bits for l in range(layers)]
    assert c["num_public"] == dense + 1 + fm
    assert c["num_constraints"] == 1 + sum(fm * _rows_per_neuron(k, shift) for k in ks) + 2 * dense
    assert c["num_variables"] == 1 + c["num_public"] + sum(fm * _vars_per_neuron(k, shift) for k in ks) + dense
    n = 1 << max(1, (c["num_constraints"] - 1).bit_length())
    mats = [c[k] for k in "ABC"]
    w_int = G._ints(c["witness"])
    assert G.first_failing_constraint(mats, w_int, c["num_constraints"], n, c["num_variables"]) == -1


def test_changed_witness_breaks_a_row():
    c = Z.synth_conv_circuit(1, 2, 4, 4, 24, 10, 0, 2, 21)
    n = 1 << (c["num_constraints"] - 1).bit_length()
    mats = [c[k] for k in "ABC"]
    w_int = G._ints(c["witness"])
    # the first conv output (first private variable): its conv row is row 1
    z = 1 + c["num_public"]
    w_int[z] = (w_int[z] + 1) % G.R
    assert G.first_failing_constraint(mats, w_int, c["num_constraints"], n, c["num_variables"]) == 1
    # a public dense output: only its equality row (the last rows) breaks
    w_int = G._ints(c["witness"])
    w_int[1] = (w_int[1] + 1) % G.R
    assert G.first_failing_constraint(mats, w_int, c["num_constraints"], n, c["num_variables"]) == \
        c["num_constraints"] - 2


def test_out_of_range_values_are_refused():
    # 8-bit ranges cannot hold a 3x3x4 int8 convolution of inputs up to 16
    with pytest.raises(Exception):
        Z.synth_conv_circuit(1, 4, 4, 4, 8, 2, 0, 1, 3)


def test_config5_shape_matches_the_reference_statement():
    c = Z.synth_conv_circuit(2, 32, 32, 32, 24, 10, 23, 10, 5)
    # the reference's statement v2 for the config-5 model: 4,128,789 constraints,
    # 4,030,486 variables, 32,779 public (10 outputs, the model tag, 32,768 inputs)
    assert c["num_constraints"] == 4_128_789
    assert c["num_variables"] == 4_030_486
    assert c["num_public"] == 32_779
    # nnz: B and C depend only on the structure; A also on which int8 weights are zero
    assert len(c["B"]) == 7_864_341 and len(c["C"]) == 131_083
    assert abs(len(c["A"]) - 26_480_000) < 0.005 * 26_480_000
    assert c["num_constraints"] <= 1 << 22 < 2 * c["num_constraints"]


def _mlp_rows(batch, n_in, n_hidden, n_out, bits, shift, context):
    per_neuron = 1 + (bits + 2) + ((shift + 1) + (bits + 1) + 1 if shift else 0)
    return 1 + (1 if context else 0) + batch * (n_hidden * per_neuron + 2 * n_out)


@pytest.mark.parametrize("args", [(4, 64, 32, 10, 24, 6, True, 1), (1, 8, 5, 3, 20, 4, False, 2), (2, 6, 4, 2, 24, 0, True, 3)])
def test_mlp_statements_are_satisfied(args):
    batch, n_in, n_hidden, n_out, bits, shift, context, seed = args
    c = Z.synth_mlp_circuit(*args)
    assert c["num_public"] == batch * n_out + 1 + (1 if context else 0) + batch * n_in
    assert c["num_constraints"] == _mlp_rows(*args[:7])
    n = 1 << max(1, (c["num_constraints"] - 1).bit_length())
    assert G.first_failing_constraint([c[k] for k in "ABC"], G._ints(c["witness"]), c["num_constraints"], n,
                                      c["num_variables"]) == -1


def test_mlp_config1_matches_the_reference_statement():
    # the reference's statement v2 for the config-1 model (batch 4 of 64 -> 32 RELU_EXACT
    # (bits 24, shift 6) -> 10, context-bound): 7,762 constraints, 7,764 variables,
    # 298 public (40 outputs, the model tag, the context, 256 inputs), domain 2^13
    c = Z.synth_mlp_circuit(4, 64, 32, 10, 24, 6, True, 1)
    assert (c["num_constraints"], c["num_variables"], c["num_public"]) == (7762, 7764, 298)
    assert 1 << 12 < c["num_constraints"] <= 1 << 13
    mats = [c[k] for k in "ABC"]
    n = 1 << 13
    # the context (public index 1 + 40 + 1) appears only in its binding row, row 1;
    # sample 0's first output only in its equality row, after the tag and context
    # rows and that sample's 32 x 60 hidden and 10 output rows
    for var, row in ((42, 1), (1, 2 + 32 * 60 + 10)):
        w = G._ints(c["witness"])
        w[var] = (w[var] + 1) % G.R
        assert G.first_failing_constraint(mats, w, c["num_constraints"], n, c["num_variables"]) == row, var


def test_mlp_out_of_range_is_refused():
    with pytest.raises(Exception):
        Z.synth_mlp_circuit(1, 64, 4, 2, 8, 2, False, 1)
