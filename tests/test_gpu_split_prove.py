"""The Groth16 prove split over devices in C (zk_groth16_prove_split /
zk_groth16_prove_multi): the proof equals the one-device proof byte for byte.

On one GPU the ranks are host threads sharing the device (zk_comm_init_local:
device copies and host barriers instead of NCCL; every kernel and layout of
the split is the same); with two or more GPUs visible, the same through NCCL
(zk_comm_init_all: one process, one host thread per device)."""
import numpy as np
import pytest

import groth16_oracle as G
import ref_statements as RS
import zkml_b200 as Z

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

CIRCUIT = (2, 4, 8, 8, 24, 10, 23, 5, 21)


@pytest.fixture(scope="module")
def key():
    c = Z.synth_conv_circuit(*CIRCUIT)
    r1 = Z.R1cs(c)
    pk = Z.ProvingKey.setup(r1, G.toxic_deterministic())
    r, s = G.blinding_deterministic()
    return c, r1, pk, r, s, pk.prove(r1, c["witness"], r, s)[0]


@pytest.mark.parametrize("nranks", [2, 4, 8])
def test_local_ranks_match_one_device(key, nranks):
    c, r1, pk, r, s, proof = key
    comms = Z.Comm.init_local(0, nranks)
    got, A, B, C, stats = Z.prove_multi([pk] * nranks, [r1] * nranks, comms, c["witness"], r, s)
    assert got == proof
    assert [st["rank"] for st in stats] == list(range(nranks))
    for st in stats:
        assert st["nranks"] == nranks and st["total_ms"] > 0 and st["compute_h_ms"] > 0 and st["all_to_all_ms"] > 0
    # a second proof through the same communicators and cached buffers
    assert Z.prove_multi([pk] * nranks, [r1] * nranks, comms, c["witness"], r, s)[0] == proof


def test_local_ranks_reference_statement():
    """Config 1's MLP statement, built by the reference's statement builder,
    split over 4 ranks: the one-device proof (itself byte-equal to the
    reference prover's, tests/test_gpu_reference_statements.py)."""
    if not RS.available():
        pytest.skip("reference statement builder not built")
    c = RS.mlp_statement()
    r1 = Z.R1cs(c)
    pk = Z.ProvingKey.setup(r1, G.toxic_deterministic())
    r, s = G.blinding_deterministic()
    comms = Z.Comm.init_local(0, 4)
    assert Z.prove_multi([pk] * 4, [r1] * 4, comms, c["witness"], r, s)[0] == pk.prove(r1, c["witness"], r, s)[0]


@pytest.mark.parametrize("nranks", [2, 4])
def test_local_ranks_refuse_unsatisfying_witness(key, nranks):
    """Every rank fails with the first failing constraint (an all-reduce MIN
    of each rank's rows), the message of the one-device prover."""
    c, r1, pk, r, s, _ = key
    w = np.array(c["witness"], copy=True)
    w[c["num_variables"] - 3] ^= np.uint64(1)
    with pytest.raises(Z.ZkError) as e1:
        pk.prove(r1, w, r, s)
    comms = Z.Comm.init_local(0, nranks)
    with pytest.raises(Z.ZkError) as e:
        Z.prove_multi([pk] * nranks, [r1] * nranks, comms, w, r, s)
    assert e.value.status == Z.ZK_ERR_INVALID
    msg = str(e1.value)
    assert msg[msg.index("[Prove]"):] in str(e.value)


def test_rank_counts_outside_the_split_are_refused(key):
    c, r1, pk, r, s, _ = key
    comms = Z.Comm.init_local(0, 3)
    with pytest.raises(Z.ZkError) as e:
        Z.prove_multi([pk] * 3, [r1] * 3, comms, c["witness"], r, s)
    assert e.value.status == Z.ZK_ERR_RANGE


def test_nccl_devices_match_one_device(key):
    ndev = torch.cuda.device_count()
    if ndev < 2:
        pytest.skip("needs two GPUs")
    c, _, _, r, s, proof = key
    nr = 4 if ndev >= 4 else 2
    r1s = [Z.R1cs(c, device=d) for d in range(nr)]
    pks = [Z.ProvingKey.setup(r1s[d], G.toxic_deterministic()) for d in range(nr)]
    comms = Z.Comm.init_all(list(range(nr)))
    got, *_ = Z.prove_multi(pks, r1s, comms, c["witness"], r, s)
    assert got == proof
