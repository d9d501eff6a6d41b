"""The reference's statement-v2 builder (oracle/_ref/libzkref_stmt.so, built
from its src/prover/statement_v2.cuh) gives the circuits of the Groth16 parity
tests with the reference's own sizes (tests/host/test_statement_v2.cpp: 8,082
and 62,692 constraints; config 1's MLP at batch 4: 7,762), satisfied by their
witnesses under the oracle's matrix-vector product, with the sizes this
library's own synthetic MLP statement reproduces."""
import numpy as np
import pytest

import pyoracle as O
import ref_statements as RS
import zkml_b200 as Z

pytestmark = pytest.mark.skipif(not RS.available(), reason="reference statement builder not built")


def _satisfied(c):
    n = c["num_constraints"]
    w = c["witness"]
    ev = []
    for k in "ABC":
        e = c[k]
        acc = [0] * n
        for row, col, v in zip(e["row"], e["col"], e["v"]):
            acc[row] = (acc[row] + O.to_int(v) * O.to_int(w[col])) % Z.R_MOD
        ev.append(acc)
    # Montgomery values: each row sum carries R^2 (entry R times witness R),
    # so (A w)(B w) carries R^4 and C w R^2
    rinv2 = pow(1 << 512, -1, Z.R_MOD)
    return all(ev[0][i] * ev[1][i] * rinv2 % Z.R_MOD == ev[2][i] for i in range(n))


@pytest.mark.parametrize("variant,nc,m,pub", [("A", 8082, 7868, 82), ("B", 62692, 62779, 8)])
def test_tiny_cnn_statement_sizes(variant, nc, m, pub):
    c = RS.tiny_cnn_statement(variant)
    assert (c["num_constraints"], c["num_variables"], c["num_public"]) == (nc, m, pub)
    assert np.array_equal(c["witness"][0], O.fr_from_int(1))
    if variant == "A":
        assert _satisfied(c)


def test_mlp_statement_matches_synthetic_sizes():
    c = RS.mlp_statement()
    s = Z.synth_mlp_circuit(4, 64, 32, 10, 24, 6, True, 1)
    assert (c["num_constraints"], c["num_variables"], c["num_public"]) == (7762, 7764, 298)
    assert (s["num_constraints"], s["num_variables"], s["num_public"]) == (7762, 7764, 298)
    assert _satisfied(c)
