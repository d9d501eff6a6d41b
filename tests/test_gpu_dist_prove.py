"""A Groth16 proof split over ranks (zkml_dist.sharded_prove) on the GPU: the
pieces behind it (row-range matvec, witness check, coset pointwise step, key
arrays, assembly) against the one-device path; the whole split with ranks as
threads of one process on one GPU, and with NCCL ranks when two GPUs are
visible; the witness check of zk_groth16_prove (R1CS::verify_witness)."""
import os
import socket
import threading

import numpy as np
import pytest

import groth16_oracle as G
import pyoracle as O
import zkml_b200 as Z
import zkml_dist as D

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CIRCUIT = (2, 4, 8, 8, 24, 10, 23, 5, 21)


@pytest.fixture(scope="module")
def key():
    c = Z.synth_conv_circuit(*CIRCUIT)
    r1 = Z.R1cs(c)
    pk = Z.ProvingKey.setup(r1, G.toxic_deterministic())
    r, s = G.blinding_deterministic()
    proof = pk.prove(r1, c["witness"], r, s)
    return c, r1, pk, r, s, proof


def _run_threads(world, c, r1, pk, r, s, witness=None):
    shared = D.ThreadComm.Shared(world)
    out = [None] * world

    def body(rank):
        try:
            torch.cuda.set_device(0)
            prover = D.CudaProver(pk, r1)
            out[rank] = D.sharded_prove(prover, D.ThreadComm(shared, rank),
                                        c["witness"] if witness is None else witness, r, s)
        except Exception as e:  # reported per rank
            out[rank] = e

    ts = [threading.Thread(target=body, args=(k,)) for k in range(world)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=600)
    return out


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_thread_ranks_match_one_device(key, world):
    c, r1, pk, r, s, proof = key
    out = _run_threads(world, c, r1, pk, r, s)
    for rank, res in enumerate(out):
        assert not isinstance(res, Exception), (rank, res)
        assert res[0] == proof[0], rank
        assert np.array_equal(res[1], proof[1]) and np.array_equal(res[2], proof[2]) and np.array_equal(res[3], proof[3])


def test_pieces_match_fused_path(key):
    c, r1, pk, r, s, proof = key
    n = 1 << r1.log_n
    w = Z.to_device(c["witness"])
    full = r1.matvec_rows(w, 0, n)
    for lo, hi in ((0, 1), (3, 517), (n - 7, n), (n // 2, n // 2)):
        part = r1.matvec_rows(w, lo, hi)
        assert torch.equal(part, full[:, lo:hi]), (lo, hi)
    # the matvec agrees with the oracle's restatement of compute_h's loops
    w_int = [O.fr_to_int(x) for x in c["witness"]]
    a_exp = G.matvec(c["A"], w_int, n, c["num_variables"])
    got = Z.to_host(full[0])
    for i in (0, 1, c["num_constraints"] - 1, n - 1):
        assert O.fr_to_int(got[i]) == a_exp[i], i
    assert Z.hadamard_check(full[0], full[1], full[2]) == -1
    # coset evaluations -> pointwise -> coset INTT equals zk_compute_h_device
    g = Z.compute_h_coset_shift(r1.log_n)
    assert O.fr_to_int(g) == G.coset_shift(r1.log_n)
    cos = [Z.ntt(Z.ntt(full[k].contiguous(), r1.log_n, True), r1.log_n, False, coset=g) for k in range(3)]
    q = Z.compute_h_pointwise(cos[0], cos[1], cos[2], r1.log_n)
    h_split = Z.ntt(q, r1.log_n, True, coset=g)
    h_fused = torch.empty_like(h_split)
    Z.check(Z.lib.zk_compute_h_device(0, Z._stream(h_fused), Z._dev_ptr(h_fused), Z._dev_ptr(full[0].contiguous()),
                                      Z._dev_ptr(full[1].contiguous()), Z._dev_ptr(full[2].contiguous()), r1.log_n))
    torch.cuda.synchronize()
    assert torch.equal(h_split, h_fused)
    arr = pk.arrays()
    assert arr["m"] == c["num_variables"] and arr["num_public"] == c["num_public"] and arr["n_h"] == n


def _corrupt(c):
    w = np.array(c["witness"], copy=True)
    victim = c["num_variables"] - 3
    w[victim] ^= np.uint64(1)
    n = G.domain(c["num_constraints"])[0]
    row = G.first_failing_constraint([c["A"], c["B"], c["C"]], [O.fr_to_int(x) for x in w], c["num_constraints"], n,
                                     c["num_variables"])
    assert row >= 0
    return w, row


def test_prove_rejects_unsatisfying_witness(key, monkeypatch):
    c, r1, pk, r, s, proof = key
    w, row = _corrupt(c)
    with pytest.raises(Z.ZkError) as ei:
        pk.prove(r1, w, r, s)
    assert ei.value.status == Z.ZK_ERR_INVALID
    assert f"constraint {row} failed" in str(ei.value)
    # the split fails the same way on every rank
    for res in _run_threads(3, c, r1, pk, r, s, witness=w):
        assert isinstance(res, Z.ZkError) and f"constraint {row} failed" in str(res), res
    # ZKML_SKIP_WITNESS_CHECK=1 proves anyway, as the reference does
    monkeypatch.setenv("ZKML_SKIP_WITNESS_CHECK", "1")
    bad_proof = pk.prove(r1, w, r, s)[0]
    assert len(bad_proof) == 256 and bad_proof != proof[0]
    # and the good witness still proves to the same bytes afterwards
    monkeypatch.delenv("ZKML_SKIP_WITNESS_CHECK")
    assert pk.prove(r1, c["witness"], r, s)[0] == proof[0]


def _free_port():
    sk = socket.socket()
    sk.bind(("127.0.0.1", 0))
    p = sk.getsockname()[1]
    sk.close()
    return p


def _nccl_worker(rank, world, port, out_dir):
    import sys
    from datetime import timedelta
    for sub in ("oracle", "cuda-zkml_b200"):
        sys.path.insert(0, os.path.join(ROOT, sub))
    import torch
    import torch.distributed as dist

    import groth16_oracle as G
    import zkml_b200 as Z
    import zkml_dist as D

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        c = Z.synth_conv_circuit(*CIRCUIT)
        r1 = Z.R1cs(c, device=rank)
        pk = Z.ProvingKey.setup(r1, G.toxic_deterministic())
        r, s = G.blinding_deterministic()
        proof = D.sharded_prove(D.CudaProver(pk, r1), D.TorchComm(), c["witness"], r, s)[0]
        open(os.path.join(out_dir, f"proof{rank}.bin"), "wb").write(proof)
        # the one-device prove on this rank's own GPU (device 1 for rank 1)
        open(os.path.join(out_dir, f"single{rank}.bin"), "wb").write(pk.prove(r1, c["witness"], r, s)[0])
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_ranks_match_one_device(key, tmp_path):
    import torch.multiprocessing as mp
    c, r1, pk, r, s, proof = key
    mp.spawn(_nccl_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for rank in range(2):
        assert open(tmp_path / f"proof{rank}.bin", "rb").read() == proof[0], rank
        assert open(tmp_path / f"single{rank}.bin", "rb").read() == proof[0], rank
