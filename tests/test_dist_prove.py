"""A Groth16 proof split over gloo ranks on CPU (zkml_dist.sharded_prove): the
oracle does each rank's device work (tests/oracle_prover.py), the ranks share
rows, polynomials and MSM slices through real torch.distributed collectives,
and the proof must be byte-identical to the one-device oracle proof.  A
witness that breaks a constraint must fail on every rank with the first
failing row, like R1CS::verify_witness."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CIRCUIT = (1, 1, 3, 3, 24, 10, 23, 2, 11)  # layers, channels, h, w, bits, shift, out_bits, dense, seed


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _circuit(kind="conv"):
    import zkml_b200 as Z
    if kind == "mlp":  # config 1's statement (7,762 constraints, domain 2^13)
        return Z.synth_mlp_circuit()
    return Z.synth_conv_circuit(*CIRCUIT)


def _worker(rank, world, port, corrupt, out_dir, kind="conv"):
    import sys
    for sub in ("oracle", "cuda-zkml_b200", "tests"):
        sys.path.insert(0, os.path.join(ROOT, sub))
    import torch.distributed as dist

    import groth16_oracle as G
    import zkml_dist as D
    from oracle_prover import OracleProver

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = _circuit(kind)
        mats = [c["A"], c["B"], c["C"]]
        pk = G.setup(mats, c["num_constraints"], c["num_variables"], c["num_public"], G.toxic_deterministic())
        w = np.array(c["witness"], copy=True)
        if corrupt is not None:
            w[corrupt] = w[corrupt] ^ np.uint64(1)  # still < r: the low limb of a reduced value
        r, s = G.blinding_deterministic()
        try:
            proof = D.sharded_prove(OracleProver(pk, mats), D.TorchComm(), w, r, s)[0]
            open(os.path.join(out_dir, f"proof{rank}.bin"), "wb").write(proof)
        except RuntimeError as e:
            open(os.path.join(out_dir, f"err{rank}.txt"), "w").write(str(e))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4])
def test_sharded_prove_matches_one_device(tmp_path, world):
    import groth16_oracle as G
    mp.spawn(_worker, args=(world, _free_port(), None, str(tmp_path)), nprocs=world, join=True)
    c = _circuit()
    mats = [c["A"], c["B"], c["C"]]
    pk = G.setup(mats, c["num_constraints"], c["num_variables"], c["num_public"], G.toxic_deterministic())
    r, s = G.blinding_deterministic()
    exp = G.prove(pk, mats, c["witness"], r, s)[0]
    for rank in range(world):
        assert open(tmp_path / f"proof{rank}.bin", "rb").read() == exp, rank


def test_sharded_prove_mlp_statement(tmp_path):
    """Config 1's MLP statement split over two gloo ranks (the split transforms at
    n = 2^13) proves to the one-device oracle proof, which verifies with the
    toxic waste known."""
    import groth16_oracle as G
    mp.spawn(_worker, args=(2, _free_port(), None, str(tmp_path), "mlp"), nprocs=2, join=True)
    c = _circuit("mlp")
    mats = [c["A"], c["B"], c["C"]]
    tox = G.toxic_deterministic()
    pk = G.setup(mats, c["num_constraints"], c["num_variables"], c["num_public"], tox)
    r, s = G.blinding_deterministic()
    exp, A, B, C, h = G.prove(pk, mats, c["witness"], r, s)
    n, log_n = G.domain(c["num_constraints"])
    at, vanish = G.qap_at_tau(mats, n, log_n, c["num_variables"], tox[0])
    pk_o = {"m": c["num_variables"], "num_public": c["num_public"], "_at": at, "_vanish": vanish, "_toxic": tox}
    assert G.trapdoor_verify(pk_o, c["witness"], r, s, h, A, B, C)
    for rank in range(2):
        assert open(tmp_path / f"proof{rank}.bin", "rb").read() == exp, rank


def test_sharded_prove_rejects_bad_witness(tmp_path):
    import groth16_oracle as G
    import pyoracle as O
    c = _circuit()
    victim = c["num_variables"] - 1  # a private wire
    mp.spawn(_worker, args=(2, _free_port(), victim, str(tmp_path)), nprocs=2, join=True)
    mats = [c["A"], c["B"], c["C"]]
    w = np.array(c["witness"], copy=True)
    w[victim] ^= np.uint64(1)
    n = G.domain(c["num_constraints"])[0]
    row = G.first_failing_constraint(mats, [O.fr_to_int(x) for x in w], c["num_constraints"], n, c["num_variables"])
    assert row >= 0
    for rank in range(2):
        msg = open(tmp_path / f"err{rank}.txt").read()
        assert f"constraint {row} failed" in msg, msg


def test_prove_plan_sizes():
    import zkml_dist as D
    s = D.prove_msm_sizes(m=10, num_public=3, l=6, n=16, n_h=16)
    assert s == {"a": 10, "b2": 10, "l": 6, "h": 16, "b1": 10}
    assert D.prove_msm_sizes(m=5, num_public=4, l=0, n=8, n_h=8)["l"] == 0
    rec = np.arange(48, dtype=np.uint64)
    assert np.array_equal(D.pack_sums(D.unpack_sums(rec)), rec)
    assert D.row_chunk(16, 3) == 6 and D.row_chunk(4, 8) == 1


def test_weighted_bounds_cover():
    import zkml_dist as D
    for n in (0, 1, 7, 1000, 3244043):
        for shares in ([1.0], [0.5, 0.5], [0.2, 0.3, 0.5], [0.0, 1.0, 0.0], [0.01] * 3 + [0.97 / 5] * 5):
            spans = [D.weighted_bounds(n, shares, r) for r in range(len(shares))]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(len(spans) - 1))
            assert all(b >= a for a, b in spans)


def test_balance_shares_moves_work_off_polynomial_owners():
    import zkml_dist as D
    # two ranks: rank 0 owns two polynomials (2 x 2.9 ms), rank 1 one; 7.7 ms of witness MSMs
    s = [0.5, 0.5]
    for _ in range(12):
        s = D.balance_shares([5.8, 2.9], [7.7 * x for x in s], s)
    assert abs(s[0] - (5.8 + 2.9 + 7.7) / 2 / 7.7 + 5.8 / 7.7) < 0.02  # poly + share * C equal on both ranks
    # eight ranks: the three owners end up with (almost) nothing
    s = [1 / 8] * 8
    for _ in range(12):
        s = D.balance_shares([2.9] * 3 + [0.0] * 5, [7.7 * x for x in s], s)
    assert max(s[:3]) < 0.01 and abs(sum(s) - 1) < 1e-9
    assert D.balance_shares([0.0], [1.0], [1.0]) == [1.0]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_split_compute_h_matches_one_device(world):
    """compute_h with every transform split over `world` thread ranks (cyclic
    re-layout, size-m transforms, all-to-alls, cross-rank steps) gives the
    one-device coefficients of h, each rank holding its blocks."""
    import threading

    import torch

    import groth16_oracle as G
    import pyoracle as O
    import zkml_dist as D
    from oracle_prover import OracleProver

    L = 8
    n = 1 << L
    rng = O.Rng(40 + world)
    abc = np.stack([rng.fr_vector(n) for _ in range(3)])
    exp = O.compute_h_from_evals(abc[0], abc[1], abc[2], L)
    pk = {"n": n, "log_n": L, "m": 1, "num_public": 0, "l": 0}
    s_log = D.split_log(world, n)
    assert s_log == world.bit_length() - 1
    m, q = n // world, n // world // world
    shared = D.ThreadComm.Shared(world, timeout=60)
    got, errs = [None] * world, []

    def run(rank):
        try:
            comm = D.ThreadComm(shared, rank)
            t = torch.from_numpy(abc[:, rank * m:(rank + 1) * m].copy().view(np.int64))
            got[rank] = D.split_compute_h(OracleProver(pk, []), comm, t, s_log).numpy().view(np.uint64)
        except Exception as e:  # surfaced below
            errs.append(e)
            shared.barrier.abort()

    ts = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errs, errs
    for rank in range(world):
        idx = [k * m + rank * q + v for k in range(world) for v in range(q)]
        assert np.array_equal(got[rank], exp[idx]), rank


def test_split_log():
    import zkml_dist as D
    assert D.split_log(1, 1 << 10) is None and D.split_log(3, 1 << 10) is None and D.split_log(16, 1 << 20) is None
    assert D.split_log(2, 4) == 1 and D.split_log(2, 2) is None and D.split_log(8, 1 << 6) == 3 and D.split_log(8, 1 << 5) is None
