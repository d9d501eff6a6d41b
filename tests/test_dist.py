"""Sharded MSM host logic with two gloo ranks on CPU: each rank computes its
slice's partial sum (the oracle stands in for the per-GPU MSM), the ranks
all-gather the 64-byte partial points and fold them with zk_g1_add_affine; the
result must equal the unsharded MSM."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, seed, g2, out_path):
    import sys
    for sub in ("oracle", "cuda-zkml_b200"):
        sys.path.insert(0, os.path.join(ROOT, sub))
    import torch.distributed as dist

    import pyoracle as O
    import zkml_b200 as Z
    import zkml_dist as D

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = O.Rng(seed)
    k = rng.fr_vector(n)
    sc = rng.fr_vector(n)
    pts = O.g2_fixed_base(k) if g2 else O.g1_fixed_base(k)
    lo, hi = D.shard_bounds(n, rank, world)
    local = O.msm_g2 if g2 else O.msm_g1
    add = Z.g2_add_affine if g2 else Z.g1_add_affine
    res = D.sharded_msm(pts[lo:hi], sc[lo:hi], local, add)
    if rank == 0:
        np.save(out_path, res)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("n,g2", [(1001, False), (3, False), (40, True)])
def test_sharded_msm_two_ranks(tmp_path, n, g2):
    import pyoracle as O
    out = str(tmp_path / "res.npy")
    mp.spawn(_worker, args=(2, _free_port(), n, 77 + n, g2, out), nprocs=2, join=True)
    rng = O.Rng(77 + n)
    k = rng.fr_vector(n)
    sc = rng.fr_vector(n)
    if g2:
        exp = O.msm_g2(O.g2_fixed_base(k), sc)
    else:
        exp = O.msm_g1(O.g1_fixed_base(k), sc)
    assert np.array_equal(np.load(out), exp)


def test_shard_bounds_cover():
    import zkml_dist as D
    for n in (0, 1, 7, 1000, 1 << 20):
        for world in (1, 2, 3, 8):
            spans = [D.shard_bounds(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
