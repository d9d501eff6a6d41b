"""Device setup + prove against the oracle's restatement of the reference's
Groth16 (oracle/groth16_oracle.py): every proving-key point and the 256-byte
proof bit-exact under the reference's deterministic seeds, the proof valid by
the trapdoor check, and the ZKMLPK3 / vk.bin writers read back by an
independent parser that is pinned to the reference's own files."""
import os

import numpy as np
import pytest

import groth16_oracle as G
import pyoracle as O
import zkml_b200 as Z
import zkmlpk3

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small():
    c = Z.synth_conv_circuit(2, 2, 4, 4, 24, 10, 23, 3, 7)
    mats = [c["A"], c["B"], c["C"]]
    tox = G.toxic_deterministic()
    pk_o = G.setup(mats, c["num_constraints"], c["num_variables"], c["num_public"], tox)
    r1 = Z.R1cs(c)
    pk = Z.ProvingKey.setup(r1, tox)
    return c, mats, tox, pk_o, r1, pk


def test_setup_matches_oracle(small, tmp_path):
    c, mats, tox, pk_o, r1, pk = small
    path = str(tmp_path / "pk.bin")
    pk.save(path)
    buf = open(path, "rb").read()
    key = zkmlpk3.parse_pk(buf)
    assert key["n"] == pk_o["n"] and key["m"] == c["num_variables"] and key["num_public"] == c["num_public"]
    assert len(buf) == zkmlpk3.pk_size(pk_o["n"], c["num_variables"], pk_o["l"])
    for name, g2 in (("A", False), ("B1", False), ("B2", True), ("L", False), ("H", False)):
        exp = pk_o[name]
        assert len(key[name]) == len(exp), name
        conv = zkmlpk3.std_g2 if g2 else zkmlpk3.std_g1
        for i in range(len(exp)):
            assert key[name][i] == conv(exp[i]), (name, i)
    for name in ("alpha1", "beta1", "delta1"):
        assert key[name] == zkmlpk3.std_g1(pk_o[name]), name
    for name in ("beta2", "gamma2", "delta2"):
        assert key[name] == zkmlpk3.std_g2(pk_o[name]), name
    assert key["tau_g2"][1] == zkmlpk3.std_g2(pk_o["tau2"])
    vk_path = str(tmp_path / "vk.bin")
    pk.save_vk(vk_path)
    vk = zkmlpk3.parse_vk(open(vk_path, "rb").read())
    assert vk["num_public"] == c["num_public"]
    assert [tuple(v) for v in vk["ic"]] == [zkmlpk3.std_g1(p) for p in pk_o["IC"]]
    assert vk["alpha1"] == zkmlpk3.std_g1(pk_o["alpha1"])


def test_prove_matches_oracle_and_verifies(small):
    c, mats, tox, pk_o, r1, pk = small
    r, s = G.blinding_deterministic()
    proof, A, B, C = pk.prove(r1, c["witness"], r, s)
    proof_o, Ao, Bo, Co, h = G.prove(pk_o, mats, c["witness"], r, s)
    assert proof == proof_o
    assert np.array_equal(A, Ao) and np.array_equal(B, Bo) and np.array_equal(C, Co)
    assert G.trapdoor_verify(pk_o, c["witness"], r, s, h, A, B, C)
    st = Z.prove_last_stats()
    assert st["total_ms"] > 0 and st["compute_h_ms"] > 0
    # proving twice with the resident key gives the same bytes
    assert pk.prove(r1, c["witness"], r, s)[0] == proof


def test_pk_file_round_trip(small, tmp_path):
    c, mats, tox, pk_o, r1, pk = small
    path = str(tmp_path / "pk.bin")
    pk.save(path)
    pk2 = Z.ProvingKey.load(path)
    r, s = G.blinding_deterministic()
    assert pk2.prove(r1, c["witness"], r, s)[0] == pk.prove(r1, c["witness"], r, s)[0]
    # fail closed on a corrupt key
    bad = str(tmp_path / "bad.bin")
    open(bad, "wb").write(b"ZKMLPK2\0" + open(path, "rb").read()[8:])
    with pytest.raises(Z.ZkError):
        Z.ProvingKey.load(bad)
    open(bad, "wb").write(open(path, "rb").read()[:1000])
    with pytest.raises(Z.ZkError):
        Z.ProvingKey.load(bad)


def test_pk_load_in_chunks_config4(tmp_path, monkeypatch):
    """A 59 MB key (129,034 variables, domain 2^18) through the chunked loader
    with 1 MiB chunks (about 60 reads overlapped with their copies):
    the loaded key proves the same bytes, records at infinity included; a file
    cut inside the last query vector is refused."""
    c = Z.synth_conv_circuit(1, 8, 16, 16, 24, 10, 0, 4, 9)
    r1 = Z.R1cs(c)
    pk = Z.ProvingKey.setup(r1, G.toxic_deterministic())
    path = str(tmp_path / "pk.bin")
    pk.save(path)
    monkeypatch.setenv("ZKML_PK_LOAD_CHUNK_MB", "1")
    pk2 = Z.ProvingKey.load(path)
    st = Z.ProvingKey.last_load_stats()
    assert st["bytes"] > (1 << 20) and st["total_ms"] > 0
    r, s = G.blinding_deterministic()
    assert pk2.prove(r1, c["witness"], r, s)[0] == pk.prove(r1, c["witness"], r, s)[0]
    raw = open(path, "rb").read()
    bad = str(tmp_path / "cut.bin")
    open(bad, "wb").write(raw[:-100])
    with pytest.raises(Z.ZkError) as e:
        Z.ProvingKey.load(bad)
    assert "truncated" in str(e.value)


def test_wrong_witness_does_not_verify(small, monkeypatch):
    """With the witness check off (ZKML_SKIP_WITNESS_CHECK=1, as the reference
    allows) a wrong witness still proves, to the oracle's bytes, and the proof
    fails the check; with the check on, the prover refuses it."""
    c, mats, tox, pk_o, r1, pk = small
    bad = c["witness"].copy()
    bad[c["num_public"] + 5] = Z.fr_from_int(7)
    r, s = 11, 13
    with pytest.raises(Z.ZkError, match="does not satisfy R1CS constraints"):
        pk.prove(r1, bad, r, s)
    monkeypatch.setenv("ZKML_SKIP_WITNESS_CHECK", "1")
    proof, A, B, C = pk.prove(r1, bad, r, s)
    proof_o, Ao, Bo, Co, h = G.prove(pk_o, mats, bad, r, s)
    assert proof == proof_o
    assert not G.trapdoor_verify(pk_o, bad, r, s, h, A, B, C)


def test_mismatched_key_is_refused(small):
    c, mats, tox, pk_o, r1, pk = small
    c2 = Z.synth_conv_circuit(1, 2, 4, 4, 24, 10, 0, 2, 9)
    r2 = Z.R1cs(c2)
    with pytest.raises(Z.ZkError):
        pk.prove(r2, c2["witness"], 3, 5)


def test_prove_2_16_config4_shape():
    """A ~60k-constraint circuit (domain 2^16, the size of the reference's config-4 statement):
    the proof passes the trapdoor check (the oracle prove would be slow here,
    so validity rather than byte equality is checked)."""
    c = Z.synth_conv_circuit(2, 4, 11, 11, 24, 10, 23, 10, 4)
    assert 1 << 15 < c["num_constraints"] <= 1 << 16
    r1 = Z.R1cs(c)
    assert r1.log_n == 16
    tox = G.toxic_deterministic()
    pk = Z.ProvingKey.setup(r1, tox)
    r, s = G.blinding_deterministic()
    proof, A, B, C = pk.prove(r1, c["witness"], r, s)
    mats = [c["A"], c["B"], c["C"]]
    n, log_n = G.domain(c["num_constraints"])
    at, vanish = G.qap_at_tau(mats, n, log_n, c["num_variables"], tox[0])
    pk_o = {"m": c["num_variables"], "num_public": c["num_public"], "_at": at, "_vanish": vanish, "_toxic": tox}
    h = G.compute_h(mats, G._ints(c["witness"]), n, log_n, c["num_variables"])
    assert G.trapdoor_verify(pk_o, c["witness"], r, s, h, A, B, C)
    # that first proof started the H-query table build and ran its H MSM without
    # the tables; once they are ready the same inputs give the same proof
    pk.precompute()
    assert pk.prove(r1, c["witness"], r, s)[0] == proof
    # the H MSM over the key's precomputed window tables (used from 2^16 points,
    # for slices of at least 3/4 of the query) equals the plain MSM over the same
    # query points, whole and in slices
    import ctypes
    import torch
    arr = pk.arrays()
    assert arr["n_h"] == 1 << 16
    d_h = Z.to_device(Z.random_fr(arr["n_h"], 77))
    d_h[5] = 0
    for lo, hi in ((0, arr["n_h"]), (3, arr["n_h"] - 5), (0, 1), (1000, 40000), (arr["n_h"] - 3, arr["n_h"]), (7, 7)):
        got = pk.h_msm(d_h, lo, hi)
        exp = np.zeros(8, np.uint64)
        if hi > lo:
            Z.check(Z.lib.zk_msm_g1_device(0, Z._stream(d_h), ctypes.c_void_p(arr["h_query"] + lo * 64),
                                           ctypes.c_void_p(d_h.data_ptr() + lo * 32), hi - lo, exp.ctypes.data_as(ctypes.c_void_p)))
        assert np.array_equal(got, exp), (lo, hi)
    torch.cuda.synchronize()


def test_h_msm_blocks_sum_to_the_whole_query():
    """The per-part H MSMs of a split proof (each part's coefficients in the
    blocks layout, over its gathered H points: window tables from 2^16 points
    per part, the plain MSM below) add up to the H MSM over the whole query."""
    import torch
    c = Z.synth_conv_circuit(2, 4, 16, 16, 24, 10, 23, 10, 6)
    r1 = Z.R1cs(c)
    assert r1.log_n == 17
    pk = Z.ProvingKey.setup(r1, G.toxic_deterministic())
    n = 1 << r1.log_n
    d_h = Z.to_device(Z.random_fr(n, 78))
    d_h[11] = 0
    whole = pk.h_msm(d_h, 0, n)
    for s_log in (1, 3):
        N = 1 << s_log
        m, q = n // N, n // N // N
        acc = np.zeros(8, np.uint64)
        for part in range(N):
            idx = torch.tensor([k * m + part * q + v for k in range(N) for v in range(q)], device=d_h.device)
            got = pk.h_msm_blocks(d_h[idx].contiguous(), s_log, part)
            acc = Z.g1_add_affine(acc, got)
        assert np.array_equal(acc, whole), s_log
    torch.cuda.synchronize()


def _device_view(ptr, rows, words):
    """A (rows, words) int64 CUDA tensor over existing device memory."""
    import torch

    class _Cai:
        def __init__(self):
            self.__cuda_array_interface__ = {"shape": (rows, words), "typestr": "<i8", "data": (int(ptr), False),
                                             "version": 3, "strides": None}
    return torch.as_tensor(_Cai(), device="cuda").clone()


def test_ceremony_random_combination_is_the_msm():
    """The phase-2 ceremony's random linear combination sum_i rho_i P_i over a
    proving key's query points (src/prover/ceremony.cuh:242-246, run here as
    the reference's own host loop from oracle/_ref) equals the MSM through the
    reference-shaped drop-in (bn254::msm_g1 records, zk_msm_g1) and through
    the device entry point, over the L and H queries of a key."""
    import ctypes

    import pyoracle as O
    if not O.ref_available():
        pytest.skip("reference arithmetic not built")
    c = Z.synth_conv_circuit(1, 2, 8, 8, 24, 10, 0, 2, 31)
    r1 = Z.R1cs(c)
    pk = Z.ProvingKey.setup(r1, G.toxic_deterministic())
    arr = pk.arrays()
    ref = O.ref()
    for name, count in (("l_query", arr["l"]), ("h_query", arr["n_h"])):
        n = min(count, 1500)
        pts = Z.to_host(_device_view(arr[name], n, 8))
        rho = O.Rng(55 + n).fr_vector(n)
        out = np.zeros(8, np.uint64)
        inf = ctypes.c_int()
        ref.ref_random_combination(O._p(out), ctypes.byref(inf), O._p(pts), O._p(rho), n)
        exp = np.zeros(8, np.uint64) if inf.value else out
        jac = Z.msm_g1_ref(Z.packed_to_ref_g1(pts), rho)
        assert np.array_equal(jac[:8] if exp.any() else np.zeros(8, np.uint64), exp), name
        assert np.array_equal(Z.msm_g1(Z.to_device(pts), Z.to_device(rho)), exp), name
