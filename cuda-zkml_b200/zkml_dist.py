"""Point-sharded MSM across ranks (one process per GPU, torch.distributed).

Each rank owns a contiguous slice of the points and scalars (its proving-key
slice stays resident on its GPU), runs the whole Pippenger pipeline locally,
and the ranks exchange only their partial sums: one affine point per rank
(64 B for G1, 128 B for G2) through an all-gather, which every rank then
folds with the host point addition.  The data path carries no collective.
"""
import numpy as np


def shard_bounds(n, rank, world):
    """[start, end) of rank's contiguous slice of n items (sizes differ by <= 1)."""
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def gather_partials(local, group=None, device=None):
    """All-gather one packed affine point per rank; returns a list of numpy
    uint64 arrays in rank order."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    t = torch.from_numpy(np.ascontiguousarray(local, dtype=np.uint64).view(np.int64))
    if device is not None:
        t = t.to(device)
    bufs = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(bufs, t, group=group)
    return [b.cpu().numpy().view(np.uint64) for b in bufs]


def combine(partials, add):
    """Fold partial affine points with `add` (zk_g1_add_affine / zk_g2_add_affine)."""
    acc = np.zeros_like(partials[0])
    for p in partials:
        acc = add(acc, p)
    return acc


def sharded_msm(points, scalars, local_msm, add, group=None, device=None):
    """sum_i s_i P_i over all ranks' slices: local_msm(points, scalars) on this
    rank's slice, all-gather of the partial points, fold with `add`."""
    return combine(gather_partials(local_msm(points, scalars), group, device), add)
