"""Work split across ranks (one process per GPU, torch.distributed).

MSM: each rank owns a contiguous slice of the points and scalars (its
proving-key slice stays resident on its GPU), runs the whole Pippenger
pipeline locally, and the ranks exchange only their partial sums: one affine
point per rank (64 B for G1, 128 B for G2) through an all-gather, which every
rank then folds with the host point addition.  The data path carries no
collective.

Groth16 prove (sharded_prove): rows of the matvec per rank; compute_h with
every transform split over the ranks (a size-n/N transform on each rank, one
all-to-all, a cross-rank step: split_compute_h); the H MSM over each rank's
own coefficients and the witness MSMs over witness slices; the partial sums
all-gathered and folded.
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


# ------------------------------------------------------------------ Groth16 prove across ranks
#
# Groth16Prover::prove (src/prover/groth16.cu:655-920) runs on device 0 only.
# Split over `world` ranks, each holding the whole proving key and circuit:
#   1. rows: rank j computes rows [j S, (j + 1) S) of A w, B w, C w (S = n /
#      world, rounded up) and checks them (R1CS::verify_witness,
#      src/prover/circuit.cuh:93-124); the first failing row is an all-reduce
#      MIN, so every rank fails the same way.
#   2. all-gather of the three evaluation vectors; polynomial k (A, B, C)
#      belongs to rank k mod world, which runs its INTT and coset NTT
#      (groth16.cu:350-363) while the other ranks start their MSM slices.
#   3. three broadcasts of the coset evaluations; every rank forms
#      (a b - c) / (g^n - 1) and the coset INTT (groth16.cu:364-383): h.
#   4. every MSM (A, B2, L, H, B1) is point-sharded over all ranks: a rank's
#      share of the witness MSMs is one slice of the witness, whose four MSMs
#      share one counting sort; the ranks all-gather their partial sums (5
#      points each) and fold them.
#   5. the proof is assembled from the five sums (groth16.cu:774-844).
# The result is byte-identical to the one-device proof: every step is exact.

MSM_ORDER = ("a", "b2", "l", "h", "b1")  # layout of the 48-word sums record
_WORDS = {"a": 8, "b2": 16, "l": 8, "h": 8, "b1": 8}
WITNESS_MSMS = ("a", "b2", "l", "b1")
_NO_ROW = np.iinfo(np.int64).max


def prove_msm_sizes(m, num_public, l, n, n_h):
    """Number of terms of each MSM of a proof (groth16.cu:776-827)."""
    num_priv = max(0, min(l, m - 1 - num_public))
    return {"a": m, "b2": m, "l": num_priv, "h": min(n, n_h), "b1": m}


def row_chunk(n, world):
    return -(-n // world)


def witness_check_enabled():
    import os
    return os.environ.get("ZKML_SKIP_WITNESS_CHECK") != "1"


def pack_sums(sums, times=()):
    """48 words of sums (A, B2, L, H, B1), then any float64 timings as their bits."""
    parts = [np.asarray(sums[k], dtype=np.uint64).reshape(-1) for k in MSM_ORDER]
    parts.append(np.asarray(times, dtype=np.float64).view(np.uint64))
    return np.concatenate(parts)


def unpack_sums(rec):
    out, o = {}, 0
    for k in MSM_ORDER:
        out[k] = rec[o:o + _WORDS[k]]
        o += _WORDS[k]
    out["times"] = np.asarray(rec[o:], dtype=np.uint64).view(np.float64)
    return out


def weighted_bounds(n, shares, rank):
    """[start, end) of rank's slice of n items when the ranks take the
    fractions `shares` (summing to 1); contiguous, covering [0, n)."""
    acc = np.concatenate([[0.0], np.cumsum(np.asarray(shares, dtype=np.float64))])
    acc /= acc[-1] if acc[-1] > 0 else 1.0
    cut = [int(round(x * n)) for x in acc]
    cut[-1] = n
    return cut[rank], cut[rank + 1]


def balance_shares(poly_s, msm_s, shares, damping=0.5, floor=0.02):
    """Fractions of the witness MSMs for the next proof.  Rank r spends poly_s[r]
    on its polynomials and msm_s[r] on its share shares[r] of the witness MSMs
    before the coset broadcasts, which wait for the slowest rank; choose new
    shares s with poly_s[r] + s_r * C equal where possible (C = sum msm_s, the
    whole witness-MSM time), s_r >= 0, and move halfway there."""
    poly = np.asarray(poly_s, dtype=np.float64)
    C = float(np.sum(msm_s))
    world = len(poly)
    if C <= 0:
        return list(shares)
    active = np.ones(world, dtype=bool)
    target = np.zeros(world)
    for _ in range(world):  # water-filling: ranks above the level take nothing
        T = (poly[active].sum() + C) / active.sum()
        target = np.where(active, (T - poly) / C, 0.0)
        if (target >= 0).all():
            break
        active &= target > 0
    target = np.clip(target, 0.0, None)
    target /= target.sum()
    new = damping * np.asarray(shares, dtype=np.float64) + (1 - damping) * target
    new /= new.sum()
    if (new >= floor).any():  # a sliver of work costs a whole MSM's fixed overhead
        new = np.where(new < floor, 0.0, new)
        new /= new.sum()
    return [float(x) for x in new]


def split_log(world, n):
    """log2(world) when compute_h's transforms split over the ranks (world a
    power of two up to 8, with world^2 <= n), else None."""
    if world < 2 or world > 8 or world & (world - 1):
        return None
    s = world.bit_length() - 1
    return s if (n >> (2 * s)) > 0 else None


def _a2a_blocks(comm, t, world):
    """All-to-all of a (k, m, 4) stack whose rows split into `world` equal
    chunks: chunk j of every vector goes to rank j; returns (k, m, 4) with the
    chunks received from rank 0, 1, ... in order."""
    k, m = t.shape[0], t.shape[1]
    send = t.reshape(k, world, m // world, 4).permute(1, 0, 2, 3).contiguous()
    recv = comm.all_to_all(send)
    return recv.permute(1, 0, 2, 3).reshape(k, m, 4).contiguous()


def _to_cyclic(comm, t, world):
    """(k, m, 4) stack of this rank's consecutive rows [rank m, rank m + m) ->
    the rows i = rank (mod world), in order (the split transforms' cyclic layout)."""
    k, m = t.shape[0], t.shape[1]
    strided = t.reshape(k, m // world, world, 4).permute(0, 2, 1, 3).contiguous()  # [k, residue, i // world]
    return _a2a_blocks(comm, strided.reshape(k, m, 4), world)


def split_compute_h(prover, comm, abc, s_log):
    """compute_h (groth16.cu:263-390) with every transform split over the
    2^s_log ranks: abc holds this rank's rows [rank m, rank m + m) of A w, B w,
    C w (m = n / world); returns this rank's m coefficients of h in the
    "blocks" layout (local k q + v = global k m + rank q + v, q = m / world).
    Each transform is a size-m transform on every rank, one all-to-all, and a
    cross-rank step (zk_ntt_cross_device); the three polynomials travel together."""
    world, rank = comm.world, comm.rank
    L = prover.log_n
    g = prover.g
    x = _to_cyclic(comm, abc, world)                                   # evaluations, cyclic
    for k in range(3):
        prover.local_ntt(x[k], L - s_log, inverse=True)
    y = _a2a_blocks(comm, x, world)
    coeffs = [prover.cross(y[k], L, s_log, rank, True, 0, g, False) for k in range(3)]    # n^-1 g^i coefficients, blocks
    z = prover.stack([prover.cross(c, L, s_log, rank, False, 1, None, False) for c in coeffs])
    del coeffs, y
    ev = _a2a_blocks(comm, z, world)                                   # coset evaluations, cyclic
    for k in range(3):
        prover.local_ntt(ev[k], L - s_log, inverse=False)
    q = prover.pointwise(ev[0], ev[1], ev[2])                          # (a b - c) / (g^n - 1), cyclic
    del ev, z
    prover.local_ntt(q, L - s_log, inverse=True)
    qb = _a2a_blocks(comm, q.reshape((1,) + tuple(q.shape)), world)[0]
    return prover.cross(qb, L, s_log, rank, True, 0, g, True)          # n^-1 g^-i coefficients, blocks


def sharded_prove(prover, comm, witness, r, s, marks=None):
    """One Groth16 proof with the work of `prover` (this rank's device) shared
    over `comm`'s ranks.  witness: (m, 4) uint64 Montgomery (host); r, s ints.
    Returns (proof bytes, A, B, C) on every rank.  `marks`: optional list that
    receives (phase, seconds) pairs, the device synchronised at each mark
    (for profiling only: it removes the overlap between phases)."""
    rank, world = comm.rank, comm.world
    mark = (lambda name: marks.append((name, prover.sync_time()))) if marks is not None else (lambda name: None)
    mark("start")
    n, m, pub = prover.n, prover.m, prover.num_public
    sizes = prove_msm_sizes(m, pub, prover.l, n, prover.n_h)
    shares = getattr(prover, "witness_shares", None)
    if shares is None or len(shares) != world:
        shares = [1.0 / world] * world
    S = row_chunk(n, world)
    lo, hi = min(n, rank * S), min(n, (rank + 1) * S)
    # every rank needs the whole witness (the matvec reads any column): each
    # uploads one slice and the slices are all-gathered over the interconnect
    Sw = row_chunk(m, world)
    wlo, whi = min(m, rank * Sw), min(m, (rank + 1) * Sw)
    w = comm.all_gather_rows(prover.pad_rows(prover.upload_witness(witness[wlo:whi]), Sw), Sw)[:m]
    mark("witness")
    abc = prover.matvec_rows(w, lo, hi)          # (3, hi - lo, 4)
    mark("matvec")
    bad = prover.check_rows(abc, lo) if witness_check_enabled() else -1
    bad = comm.all_reduce_min(bad if bad >= 0 else _NO_ROW, like=w)
    mark("check")
    if bad != _NO_ROW:
        raise prover.error(f"[Prove] Witness does not satisfy R1CS constraints (constraint {bad} failed)")
    s_log = split_log(world, n)
    if s_log is not None:
        # every transform of compute_h split over the ranks, then the H MSM over
        # each rank's own coefficients; the witness MSMs need only the witness and
        # run beside them (their bucket fixups and reductions are chains of
        # dependent additions that leave most of the device idle)
        a, b = weighted_bounds(m, shares, rank)
        side = prover.start_witness_msms(w, a, b, overlap=marks is None)
        t_poly = prover.timer()
        h_part = split_compute_h(prover, comm, prover.stack([prover.pad_rows(abc[k], S) for k in range(3)]), s_log)
        t_poly = prover.elapsed(t_poly)
        del abc
        mark("h")
        h_sum = prover.h_msm_blocks(h_part, s_log, rank) if sizes["h"] > 0 else np.zeros(8, np.uint64)
        mark("h_msm")
        rec, t_msm = side()
        sums = unpack_sums(rec)
        sums["h"] = h_sum
        mark("witness_msms")
        return _finish(prover, comm, r, s, sums, shares, t_poly, t_msm, mark)
    full = [comm.all_gather_rows(prover.pad_rows(abc[k], S), S)[:n] for k in range(3)]
    mark("gather")
    owners = [k % world for k in range(3)]
    t_poly = prover.timer()
    cosets = [prover.to_coset(full[k]) if owners[k] == rank else prover.empty_vector() for k in range(3)]
    t_poly = prover.elapsed(t_poly)
    del full, abc
    mark("cosets")

    # the witness MSMs come before the broadcasts, which wait for the slowest
    # polynomial owner: owners take smaller slices of the witness (balance_shares)
    t_msm = prover.timer()
    a, b = weighted_bounds(m, shares, rank)
    sums = unpack_sums(prover.witness_msms(w, a, b))
    t_msm = prover.elapsed(t_msm)
    mark("witness_msms")
    for k in range(3):
        comm.broadcast(cosets[k], owners[k])
    mark("broadcast")
    h = prover.h_from_cosets(*cosets)
    del cosets
    mark("h")
    a, b = shard_bounds(sizes["h"], rank, world)
    sums["h"] = prover.msm("h", a, b, h, 0)
    mark("h_msm")
    return _finish(prover, comm, r, s, sums, shares, t_poly, t_msm, mark)


def _finish(prover, comm, r, s, sums, shares, t_poly, t_msm, mark):
    """All-gather the partial sums (and timings), rebalance the witness slices
    for the next proof, assemble."""
    recs = comm.all_gather_points(pack_sums(sums, (t_poly(), t_msm())))
    parts = [unpack_sums(p) for p in recs]
    prover.witness_shares = balance_shares([p["times"][0] for p in parts], [p["times"][1] for p in parts], shares)
    out = prover.assemble_parts(r, s, [np.asarray(p, dtype=np.uint64)[:48] for p in recs])
    mark("assemble")
    return out


class TorchComm:
    """Collectives over torch.distributed (NCCL for CUDA tensors, gloo for CPU)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist, self.group = dist, group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)

    def all_reduce_min(self, value, like):
        import torch
        t = torch.tensor([value], dtype=torch.int64, device=like.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MIN, group=self.group)
        return int(t.item())

    def all_gather_rows(self, local, chunk):
        import torch
        out = torch.empty((self.world * chunk,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        self.dist.all_gather_into_tensor(out, local.contiguous(), group=self.group)
        return out

    def broadcast(self, t, src):
        self.dist.broadcast(t, src, group=self.group)
        return t

    def all_to_all(self, t):
        """t: (world, ...) contiguous; slice j goes to rank j; returns the
        slices received, in rank order."""
        out = t.new_empty(t.shape)
        self.dist.all_to_all_single(out, t.contiguous(), group=self.group)
        return out

    def all_gather_points(self, rec):
        import torch
        dev = None
        if self.dist.get_backend(self.group) == "nccl":
            dev = torch.device("cuda", torch.cuda.current_device())
        return gather_partials(rec, self.group, dev)


class ThreadComm:
    """Ranks as threads of one process (sharing one device): an exact
    stand-in for the collectives, for testing the split on a single GPU."""

    class Shared:
        def __init__(self, world, timeout=300.0):
            import threading
            self.world = world
            self.barrier = threading.Barrier(world, timeout=timeout)
            self.slots = [None] * world

    def __init__(self, shared, rank):
        self.sh, self.rank, self.world = shared, rank, shared.world

    def _exchange(self, item):
        self.sh.slots[self.rank] = item
        self.sh.barrier.wait()
        items = list(self.sh.slots)
        self.sh.barrier.wait()
        return items

    @staticmethod
    def _sync(t):
        import torch
        if t is not None and t.is_cuda:
            torch.cuda.current_stream(t.device).synchronize()

    def all_reduce_min(self, value, like):
        return min(self._exchange(int(value)))

    def all_gather_rows(self, local, chunk):
        import torch
        self._sync(local)
        items = self._exchange(local)
        out = torch.cat([x.to(local.device) for x in items])
        self._sync(out)  # the other ranks' buffers stay untouched until this copy is done
        self.sh.barrier.wait()
        return out

    def broadcast(self, t, src):
        self._sync(t)
        items = self._exchange(t if self.rank == src else None)
        if self.rank != src:
            t.copy_(items[src])
            self._sync(t)
        return t

    def all_gather_points(self, rec):
        return self._exchange(np.array(rec, copy=True))

    def all_to_all(self, t):
        import torch
        self._sync(t)
        items = self._exchange(t)
        out = torch.stack([x[self.rank].to(t.device) for x in items])
        self._sync(out)  # the other ranks' buffers stay untouched until this copy is done
        self.sh.barrier.wait()
        return out


class CudaProver:
    """This rank's device work for sharded_prove, through the C ABI
    (key and circuit resident on one device)."""

    def __init__(self, pk, r1cs):
        import zkml_b200 as Z
        self.Z, self.pk, self.r1cs = Z, pk, r1cs
        self.arr = pk.arrays()
        self.device = self.arr["device"]
        self.m, self.num_public, self.l, self.n_h = self.arr["m"], self.arr["num_public"], self.arr["l"], self.arr["n_h"]
        self.log_n = r1cs.log_n
        self.n = 1 << r1cs.log_n
        self.g = Z.compute_h_coset_shift(self.log_n)
        self._pinned = None

    def error(self, msg):
        return self.Z.ZkError(self.Z.ZK_ERR_INVALID, msg)

    def upload_witness(self, witness):
        """Host witness -> device.  A witness already in pinned memory is copied
        straight from it; otherwise it is staged through a pinned buffer."""
        import torch
        witness = np.ascontiguousarray(witness, dtype=np.uint64)
        src = torch.from_numpy(witness.view(np.int64))
        if not src.is_pinned():
            if self._pinned is None or self._pinned.shape[0] != witness.shape[0]:
                self._pinned = torch.empty((witness.shape[0], 4), dtype=torch.int64, pin_memory=True)
            self._pinned.copy_(src)
            src = self._pinned
        return src.to(torch.device("cuda", self.device), non_blocking=True)

    def sync_time(self):
        import time

        import torch
        torch.cuda.synchronize(self.device)
        return time.perf_counter()

    def timer(self):
        """Start a device-time measurement on the current stream."""
        import torch
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def elapsed(self, start):
        """Stop it; returns a callable giving the seconds, read once the work is done."""
        import torch
        end = torch.cuda.Event(enable_timing=True)
        end.record()

        def read():
            end.synchronize()
            return start.elapsed_time(end) / 1e3
        return read

    def matvec_rows(self, w, lo, hi):
        return self.r1cs.matvec_rows(w, lo, hi)

    def check_rows(self, abc, row0):
        if abc.shape[1] == 0:
            return -1
        return self.Z.hadamard_check(abc[0], abc[1], abc[2], row0)

    def pad_rows(self, v, rows):
        import torch
        if v.shape[0] == rows:
            return v
        out = torch.zeros((rows, 4), dtype=v.dtype, device=v.device)
        out[:v.shape[0]] = v
        return out

    def empty_vector(self):
        import torch
        return torch.empty((self.n, 4), dtype=torch.int64, device=torch.device("cuda", self.device))

    def to_coset(self, v):
        """Evaluations on the domain -> evaluations on the coset g H."""
        coeffs = self.Z.ntt(v.contiguous(), self.log_n, inverse=True)
        return self.Z.ntt(coeffs, self.log_n, inverse=False, coset=self.g, out=coeffs)

    def h_from_cosets(self, a, b, c):
        q = self.Z.compute_h_pointwise(a, b, c, self.log_n)
        return self.Z.ntt(q, self.log_n, inverse=True, coset=self.g, out=q)

    def witness_msms(self, w, lo, hi):
        return self.pk.witness_msms(w, lo, hi)

    def start_witness_msms(self, w, lo, hi, overlap=True):
        """The witness MSMs over [lo, hi) from a host thread on a side stream
        (ordered after the work already queued for w), beside the caller's
        work on its own stream; returns a callable giving (sums record, device
        seconds) once they are done.  overlap=False runs them here and now."""
        import threading

        import torch
        if not overlap:
            t = self.timer()
            rec = self.witness_msms(w, lo, hi)
            el = self.elapsed(t)
            return lambda: (rec, el)
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(device=self.device)
        ready = torch.cuda.Event()
        ready.record()
        box = {}

        def body():
            try:
                torch.cuda.set_device(self.device)
                with torch.cuda.stream(self._side):
                    self._side.wait_event(ready)
                    t = self.timer()
                    box["rec"] = self.witness_msms(w, lo, hi)
                    box["el"] = self.elapsed(t)
            except BaseException as e:  # re-raised by the caller
                box["err"] = e

        th = threading.Thread(target=body)
        th.start()

        def finish():
            th.join()
            if "err" in box:
                raise box["err"]
            torch.cuda.current_stream(self.device).wait_stream(self._side)
            w.record_stream(self._side)
            return box["rec"], box["el"]
        return finish

    def stack(self, vs):
        import torch
        return torch.stack(list(vs))

    def local_ntt(self, v, log_m, inverse):
        """In place: this rank's size-2^log_m share of a split transform."""
        self.Z.ntt(v, log_m, inverse=inverse, out=v)

    def cross(self, v, log_n, s_log, part, inverse, mode, factor, factor_inverse):
        return self.Z.ntt_cross(v, log_n, s_log, part, inverse, mode, factor, factor_inverse)

    def pointwise(self, a, b, c):
        return self.Z.compute_h_pointwise(a, b, c, self.log_n)

    def h_msm_blocks(self, h_part, s_log, part):
        return self.pk.h_msm_blocks(h_part, s_log, part)

    def msm(self, key, lo, hi, scalars, scalar_offset):
        import ctypes
        words = _WORDS[key]
        out = np.zeros(words, np.uint64)
        if hi <= lo:
            return out
        if key == "h" and scalar_offset == 0:  # over the key's precomputed H tables
            return self.pk.h_msm(scalars, lo, hi)
        base = {"a": "a", "b2": "b2", "l": "l_query", "h": "h_query", "b1": "b1"}[key]
        rec = 128 if key == "b2" else 64
        pts = ctypes.c_void_p(self.arr[base] + lo * rec)
        sc = ctypes.c_void_p(scalars.data_ptr() + (scalar_offset + lo) * 32)
        fn = self.Z.lib.zk_msm_g2_device if key == "b2" else self.Z.lib.zk_msm_g1_device
        self.Z.check(fn(self.device, self.Z._stream(scalars), pts, sc, hi - lo, out.ctypes.data_as(ctypes.c_void_p)))
        return out

    def add_g1(self, a, b):
        return self.Z.g1_add_affine(a, b)

    def add_g2(self, a, b):
        return self.Z.g2_add_affine(a, b)

    def assemble(self, r, s, sums):
        return self.pk.assemble(r, s, sums)

    def assemble_parts(self, r, s, parts):
        return self.pk.assemble_parts(r, s, parts)
