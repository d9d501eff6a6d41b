"""bench.py -- G1 MSM points/s at 2^24 points per GPU (the headline metric, on
the standalone-MSM benchmark configuration) on B200, one process per GPU.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--log-n L] [--impl b200|reference]

A step is one full G1 Pippenger MSM of the rank's 2^L-point shard (uniform
254-bit Fr scalars, points k_i * G1 for seeded uniform k_i, generated on the
device) plus, for N > 1, the all-gather of the per-rank partial points and
their fold on every rank (the sharded MSM of N * 2^L points; weak scaling).

value : points/s over all ranks with inputs resident in HBM (1.5 GiB per rank,
        larger than the 126 MB L2, so no flush is needed between steps).
e2e   : the same MSM through the host-buffer entry point zk_msm_g1_host, with
        the points and scalars copied from pinned host memory every step and
        the result read back to the host.
roofline: the bucket-accumulation kernel (the dominant one) against the
        hardware issue rate of mad.lo.u32 on this GPU, measured in the run
        (zk_probe_int_pipe); the fractions against a lo/hi product pair and
        against the library's own Montgomery multiplication ride along.
cpu_baseline: the oracle's multi-threaded Pippenger (a CPU restatement of the
        reference's algorithm) on a 2^18-point sample of the same inputs.
--impl reference: the reference's Pippenger schedule (src/msm/msm.cu) with its
        own host arithmetic (compiled from its sources into oracle/_ref) on all
        host cores, over a 2^18-point sample per step; beside it, the
        reference's own GPU NTT (bn254::ntt_gpu built for sm_100a) at 2^16,
        2^20 and 2^24 on the same B200, and the reference's Groth16Prover::prove
        linked against this library on configs 1 and 4.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cuda-zkml_b200"))

R_MOD = 21888242871839275222246405745257275088548364400416034343698204186575808495617
METRIC = "G1 MSM points/s @2^24"


def msm_ref_ops(n):
    """Algorithmic Fp multiplications of the reference's Pippenger at n points:
    11 n W + 32 W (2^c - 1) with (c, W) = MSMConfig::for_size(n)."""
    c = 10 if n <= 1 << 10 else 12 if n <= 1 << 14 else 14 if n <= 1 << 18 else 15 if n <= 1 << 22 else 16
    W = (253 + c) // c
    return 11 * n * W + 32 * W * ((1 << c) - 1)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = [r.split(",") for r in (self.out or "").strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def emit(obj):
    print(json.dumps(obj), flush=True)


def host_cpu():
    """The host the CPU figures ran on: logical cores and the CPU model name."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"nproc": os.cpu_count(), "model": model}


# ---------------------------------------------------------------- reference arm
def reference_gpu_ntt(ref, sizes, reps=3):
    """The reference's own GPU NTT entry point bn254::ntt_gpu (src/ntt/ntt.cu:
    354-465, compiled for sm_100a from its source into oracle/_ref/libzkref.so)
    on this B200: wall time of the synchronous call (it allocates, builds each
    global stage's twiddles on the host and copies them, as a reference user
    gets it), device buffers allocated here.  No lock or wait in its kernels."""
    import torch
    out = {}
    dev = torch.device("cuda", 0)
    for ln in sizes:
        n = 1 << ln
        x = torch.randint(0, 1 << 62, (n, 4), dtype=torch.int64, device=dev)
        x[:, 3] &= (1 << 60) - 1  # below r
        y = torch.empty_like(x)
        ref.ref_ntt_gpu(ctypes_ptr(y), ctypes_ptr(x), ln, 0)  # warm-up
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(reps):
            ref.ref_ntt_gpu(ctypes_ptr(y), ctypes_ptr(x), ln, 0)
        torch.cuda.synchronize()
        out[f"2^{ln}"] = {"ms": 1e3 * (time.perf_counter() - t0) / reps, "reps": reps}
        del x, y
    return out


def reference_drop_in_prove(reps=3):
    """The reference's own Groth16Prover::prove (src/prover/groth16.cu:655-920)
    linked against this library's bn254::msm_g1 / msm_g2 / ntt_gpu
    (oracle/_ref/libzkref_g16.so): what a zkml-prove user gets from swapping the
    library in.  Configs 1 and 4 as the reference's build_statement_v2 builds
    them, keys from this library's setup under the reference's deterministic
    toxic waste, loaded by the reference from ZKMLPK3 files; the time is the
    prove call alone (its host matvec, witness check and PCIe round trips
    included), beside zk_groth16_prove on the same key and witness.  Every
    proof is checked equal to this library's."""
    import tempfile
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import groth16_oracle as G
    import ref_statements as RS
    import zkml_b200 as Z
    for p in (RS.STMT_LIB, RS.G16_LIB):
        if not os.path.exists(p):
            return {"unavailable": f"{os.path.basename(p)} not built"}
    lib = RS.g16(RS.G16_LIB)
    out = {}
    for name, build in (("config1_mlp_b4", RS.mlp_statement), ("config4_statement_v2_B", lambda: RS.tiny_cnn_statement("B"))):
        c = build()
        r1 = Z.R1cs(c)
        pk = Z.ProvingKey.setup(r1, G.toxic_deterministic())
        r, s = G.blinding_deterministic()
        with tempfile.TemporaryDirectory() as d:
            pk_path, vk_path = os.path.join(d, "pk.bin"), os.path.join(d, "vk.bin")
            pk.save(pk_path)
            pk.save_vk(vk_path)
            ours, ref_ms, our_ms = None, [], []
            for _ in range(reps + 1):
                t0 = time.perf_counter()
                ours = pk.prove(r1, c["witness"], r, s)[0]
                our_ms.append(1e3 * (time.perf_counter() - t0))
                proof, ok, ms = RS.prove_with_keys(lib, pk_path, vk_path, c)
                if not ok or proof != ours:
                    return {"error": f"{name}: the drop-in proof differs or fails to verify"}
                ref_ms.append(ms)
        out[name] = {"constraints": c["num_constraints"], "log_n": r1.log_n,
                     "reference_prove_ms": statistics.median(ref_ms[1:]),
                     "zk_groth16_prove_ms": statistics.median(our_ms[1:]), "reps": reps, "proofs_equal": True}
        del pk, r1
    return out


def ctypes_ptr(t):
    import ctypes
    return ctypes.c_void_p(t.data_ptr())


def run_reference(args):
    """The reference's CPU MSM path at this workload: its Pippenger schedule
    (src/msm/msm.cu:320-442: MSMConfig windows, unsigned digits, add_affine
    buckets, running-sum reduce, host combine) executed on the host cores with
    its own host arithmetic (src/field, src/curve compiled from its sources into
    oracle/_ref), on a bounded sample of the 2^L points per step.  Its GPU MSM
    is not run (unbounded atomicCAS spin locks, msm.cu:63-72); its GPU NTT is
    timed beside it on the same B200."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ctypes

    import pyoracle as O

    cores = os.cpu_count() or 1
    n = args.ref_sample
    rng = O.Rng(0x5EED0000 + args.log_n)
    k = rng.fr_vector(n)
    pts = O.g1_fixed_base(k)
    sc = rng.fr_vector(n)
    out = np.zeros(8, np.uint64)
    inf = ctypes.c_int()
    gpu_ntt = drop_in = None
    if O.ref_available():
        ref = O.ref()
        kind = "reference"

        def step():
            ref.ref_msm_g1_pippenger_mt(O._p(out), ctypes.byref(inf), O._p(pts), O._p(sc), n, cores)
        what = ("reference Pippenger schedule (src/msm/msm.cu:320-442) with the reference's own host arithmetic "
                "(src/field, src/curve), windows split over the host threads")
        if not args.no_ntt:
            try:
                import torch
                if torch.cuda.is_available():
                    ref.ref_ntt_gpu.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
                    gpu_ntt = reference_gpu_ntt(ref, (16, 20, 24))
            except Exception as e:  # reported, not fatal: the MSM arm stands alone
                gpu_ntt = {"error": str(e)[:200]}
        if not args.no_prove:
            try:
                import torch
                if torch.cuda.is_available():
                    drop_in = reference_drop_in_prove()
            except Exception as e:
                drop_in = {"error": str(e)[:200]}
    else:
        kind = "port"

        def step():
            out[:] = O.msm_g1(pts, sc, nthreads=cores)
        what = "oracle restatement of the reference Pippenger (oracle/bn254_oracle.c)"
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = n / dt
    naive = None
    if kind == "reference":
        # for context: the sum of scalar_mul of the reference's CPU test helper
        # (tests/test_msm.cu:20-28) and of msm_g1's small-n path (src/msm/
        # msm.cu:330-339), with its host arithmetic, at 2^16 points on all cores
        nn = 1 << 16
        t0 = time.perf_counter()
        ref.ref_msm_g1_naive_mt(O._p(out), ctypes.byref(inf), O._p(pts[:nn]), O._p(sc[:nn]), nn, cores)
        nt = time.perf_counter() - t0
        naive = {"points": nn, "ms": nt * 1e3, "points_per_s": nn / nt, "cores": cores}
    sample = f"{n} of the 2^{args.log_n} points per step, {what}, {cores} threads"
    emit({"impl": "reference", "metric": METRIC, "value": value, "unit": "points/s", "n_gpus": args.gpus,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
          "scaling": "weak", "vs_baseline": None, "dtype": "u32", "data": "synthetic",
          "config": {"workload": f"G1 MSM, 2^{args.log_n} points per GPU (configs[1])", "log_n": args.log_n,
                     "sample_points": n},
          "cpu_baseline": {"value": value, "unit": "points/s", "cores": cores, "kind": kind, "sample": sample, "host": host_cpu()},
          "e2e": {"value": value, "unit": "points/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
          "reference_gpu_ntt": gpu_ntt, "reference_drop_in_prove": drop_in, "reference_naive_msm": naive})


# ---------------------------------------------------------------- Groth16 prove
def bench_prove(Z, args, dev, world=1, rank=0):
    """Groth16 prove of the synthetic statement of the large prove configuration
    (2 x [CONV 3x3, 32 ch, 32x32, RELU_EXACT with bit-decomposed range checks,
    widths 24 then 23, shift 10] + dense 32768 -> 10 with public outputs;
    4,128,789 constraints, domain 2^22), proving key from the device
    setup under the reference's deterministic toxic waste, key and circuit
    resident; a step is one prove from the host witness to the 256-byte proof.
    With world > 1 every rank holds the key and the proof is split over the
    ranks (zkml_dist.sharded_prove); the step time is the max over ranks of
    CUDA-event time around the whole prove."""
    import torch
    if world > 1:
        return bench_prove_sharded(Z, args, dev, world, rank)
    c = Z.synth_conv_circuit(2, args.prove_channels, args.prove_hw, args.prove_hw, 24, 10, 23, 10, 5)
    r1 = Z.R1cs(c, device=dev.index)
    t0 = time.perf_counter()
    mt = np.random.default_rng(0)  # toxic waste is only an input here; its distribution does not matter
    tox = tuple(int(x) for x in mt.integers(1, 2**63, size=5))
    pk = Z.ProvingKey.setup(r1, tox)
    setup_s = time.perf_counter() - t0
    # the witness arrives in pinned host memory, as a prover service would stage it
    w_pin = torch.empty((c["num_variables"], 4), dtype=torch.int64, pin_memory=True)
    w_pin.copy_(torch.from_numpy(c["witness"].view(np.int64)))
    w = w_pin.numpy().view(np.uint64)
    pk.precompute()  # the H-query tables (else the first proofs run without them while they build)
    for _ in range(2):
        pk.prove(r1, w, 12345, 67890)
    torch.cuda.synchronize()
    times = []
    for _ in range(args.prove_steps):
        t0 = time.perf_counter()
        pk.prove(r1, w, 12345, 67890)
        times.append(time.perf_counter() - t0)
    st = Z.prove_last_stats()
    # cold start: the key written as ZKMLPK3 and loaded back (chunked reads into
    # pinned memory, records unpacked to Montgomery form on the GPU), then the
    # first proof with it (which also builds the H-query window tables)
    cold = None
    if not args.no_cold:
        import tempfile
        with tempfile.TemporaryDirectory() as td:
            path = os.path.join(td, "pk.bin")
            pk.save(path)
            size = os.path.getsize(path)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            pk2 = Z.ProvingKey.load(path, device=dev.index)
            load_s = time.perf_counter() - t0
            ls = Z.ProvingKey.last_load_stats()
            t0 = time.perf_counter()
            first = pk2.prove(r1, w, 12345, 67890)[0]
            first_s = time.perf_counter() - t0
            t0 = time.perf_counter()
            pk2.precompute()  # waits for the table build the first proof started as it ended
            tables_s = time.perf_counter() - t0
            t0 = time.perf_counter()
            second = pk2.prove(r1, w, 12345, 67890)[0]
            warm_s = time.perf_counter() - t0
            cold = {"pk_bytes": size, "load_ms": load_s * 1e3, "load_read_ms": ls["read_ms"], "load_alloc_ms": ls["alloc_ms"],
                    "load_call_ms": ls["total_ms"], "first_prove_ms": first_s * 1e3,
                    "cold_total_ms": (load_s + first_s) * 1e3, "tables_ready_after_ms": tables_s * 1e3,
                    "warm_prove_ms": warm_s * 1e3,
                    "proofs_equal": first == second == pk.prove(r1, w, 12345, 67890)[0],
                    "what": ("ZKMLPK3 file (page cache) -> device key -> first proof (its H MSM without tables, "
                             "whose build it starts as it ends) -> wait for the tables -> a warm proof")}
            del pk2
    # the timed proof checks out: this library's verifier (pairing on the host,
    # public-input MSM over the 32,779 IC points on the GPU)
    proof = pk.prove(r1, w, 12345, 67890)[0]
    vk = Z.VerifyingKey.from_pk(pk)
    pub = np.ascontiguousarray(w[1:1 + c["num_public"]])
    t0 = time.perf_counter()
    verified = vk.verify(pub, proof, device=dev.index)
    verify_ms = 1e3 * (time.perf_counter() - t0)
    bad = bytearray(proof)
    bad[70] ^= 1
    tampered_rejected = not vk.verify(pub, bytes(bad), device=dev.index)
    return {"config": f"synthetic statement: 2 x CONV2D 3x3 {args.prove_channels}ch {args.prove_hw}x{args.prove_hw} + RELU_EXACT, dense 10 (config 5)",
            "proof_verifies": bool(verified), "tampered_proof_rejected": bool(tampered_rejected), "verify_ms": verify_ms,
            "cold_start": cold,
            "constraints": c["num_constraints"], "variables": c["num_variables"], "public": c["num_public"],
            "nnz": [len(c["A"]), len(c["B"]), len(c["C"])], "log_n": r1.log_n,
            "prove_ms": 1e3 * statistics.median(times), "prove_ms_min": 1e3 * min(times), "steps": args.prove_steps,
            "setup_s": setup_s, "device_phases_ms": st,
            "timed": "host witness in -> 256-byte proof out; proving key and R1CS resident on the device (warm)"}


def bench_prove_sharded(Z, args, dev, world, rank):
    """The proof split over the ranks by the library's C split prover
    (zk_groth16_prove_split over an NCCL communicator made from an id that rank 0
    broadcasts; nothing of torch inside the timed call): witness slices
    all-gathered, matvec rows and witness check per rank, every compute_h
    transform split (size-n/N NTT + one all-to-all + cross-rank N-point step),
    the H MSM over each rank's coefficients, the witness MSMs over witness slices
    beside it, partial sums all-gathered.  The step time is the max over ranks of
    the call's time; per-rank phase times come from zk_groth16_split_last_stats."""
    import torch
    import torch.distributed as dist
    if world & (world - 1) or world > 8:
        return {"skipped": f"the split prove takes a power of two up to 8 ranks, not {world}"}
    c = Z.synth_conv_circuit(2, args.prove_channels, args.prove_hw, args.prove_hw, 24, 10, 23, 10, 5)
    r1 = Z.R1cs(c, device=dev.index)
    t0 = time.perf_counter()
    mt = np.random.default_rng(0)
    tox = tuple(int(x) for x in mt.integers(1, 2**63, size=5))
    pk = Z.ProvingKey.setup(r1, tox)
    setup_s = time.perf_counter() - t0
    w_pin = torch.empty((c["num_variables"], 4), dtype=torch.int64, pin_memory=True)
    w_pin.copy_(torch.from_numpy(c["witness"].view(np.int64)))
    w = w_pin.numpy().view(np.uint64)
    uid = [Z.Comm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    comm = Z.Comm.init_rank(dev.index, uid[0], world, rank)
    for _ in range(3):
        proof = Z.prove_split(pk, r1, comm, w, 12345, 67890)[0]
    # parity: the split proof equals this rank's one-device proof
    same = proof == pk.prove(r1, w, 12345, 67890)[0]
    flag = torch.tensor([1 if same else 0], dtype=torch.int64, device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    times, stats = [], []
    for _ in range(args.prove_steps):
        dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        res = Z.prove_split(pk, r1, comm, w, 12345, 67890)
        e1.record()
        torch.cuda.synchronize()
        stats.append(res[4])
        t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times.append(float(t.item()) / 1e3)
    best = min(range(len(times)), key=lambda i: times[i])
    mine = {k: round(v, 3) for k, v in stats[best].items() if k not in ("nranks", "rank")}
    per_rank = [None] * world
    dist.all_gather_object(per_rank, mine)
    del comm
    return {"config": f"synthetic statement: 2 x CONV2D 3x3 {args.prove_channels}ch {args.prove_hw}x{args.prove_hw} + RELU_EXACT, dense 10 (config 5)",
            "phase_ms_per_rank": per_rank,
            "constraints": c["num_constraints"], "variables": c["num_variables"], "public": c["num_public"],
            "nnz": [len(c["A"]), len(c["B"]), len(c["C"])], "log_n": r1.log_n,
            "prove_ms": 1e3 * statistics.median(times), "prove_ms_min": 1e3 * min(times), "steps": args.prove_steps,
            "setup_s": setup_s, "n_gpus": world, "proof_equals_one_device": bool(flag.item()),
            "api": "zk_groth16_prove_split (C, NCCL communicator from zk_comm_init_rank)",
            "parallelism": ("witness slices all-gathered, matvec rows + witness check per rank, every compute_h transform "
                            "split over the ranks (size-n/N NTT + NCCL grouped send/recv all-to-all + cross-rank N-point step), "
                            "H MSM over each rank's coefficients, witness MSMs over witness slices beside it, partial sums "
                            "all-gathered"),
            "timed": "host witness in -> 256-byte proof out on every rank; max over ranks of the call's time"}


# ---------------------------------------------------------------- B200 arm
def run_b200(args):
    import torch
    import torch.distributed as dist

    import zkml_b200 as Z
    import zkml_dist as D

    world, rank, local = dist_env()
    if world != args.gpus:
        args.gpus = world
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    n = 1 << args.log_n
    # inputs: this rank's shard of the global N * 2^L-point MSM
    k = Z.random_fr(n, 0x5EED0000 + args.log_n + 1000 * rank)
    sc = Z.random_fr(n, 0x5EED8000 + args.log_n + 1000 * rank)
    pts_d = Z.g1_fixed_base(Z.to_device(k, dev))
    sc_d = Z.to_device(sc, dev)
    del k
    torch.cuda.synchronize()

    def reduce_max(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def step_device():
        part = Z.msm_g1(pts_d, sc_d)
        if world > 1:
            part = D.combine(D.gather_partials(part, device=dev), Z.g1_add_affine)
        return part

    imad = max(Z.probe_imad_rate(local) for _ in range(3))  # the library's own multiplication, 256 IMAD each
    pipe = max((Z.probe_int_pipe(local) for _ in range(2)), key=lambda r: r["mad_lo_per_s"])
    hw_peak = pipe["mad_lo_per_s"]  # hardware mad.lo.u32 issue rate at the clock this run sees

    for _ in range(args.warmup):
        step_device()
    stats = []
    sampler = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with sampler:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step_device()
            stats.append(Z.msm_last_stats())
        e1.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = reduce_max(e0.elapsed_time(e1) / args.steps)
    value = world * n / (ms / 1e3)

    acc_ms = reduce_max(statistics.mean(s["accumulate_ms"] for s in stats))
    adds = stats[-1]["bucket_adds"]
    launches = stats[-1]["kernel_launches"] * args.steps
    # algorithmic IMAD of the accumulate kernel: bucket_adds mixed XYZZ additions,
    # each 8M + 2S.  On 8 x 32-bit limbs a product is 128 product + 128 reduction
    # multiply-adds; a squaring 72 + 128 (each cross product once); the two products
    # of Y3 = R (Q - X3) - Y1 PPP share one reduction (256 + 128).  Per addition:
    # 6 x 256 + 2 x 200 + 384 = 2320 IMAD.
    imad_per_add = 6 * 256 + 2 * 200 + 384
    # With the batch-affine rounds (G1, full buckets) most of the additions are
    # affine pair additions sharing one inversion per round: 5 products + 1
    # squaring each (3 for the shared inversion, the slope, y3; the squared
    # slope): 5 x 256 + 200 = 1480 IMAD; the elements they leave go through the
    # mixed XYZZ additions above (counted as if every one were an addition).
    imad_per_pair = 5 * 256 + 200
    ba_pairs = stats[-1].get("batch_affine_pairs", 0)
    ba_left = stats[-1].get("batch_affine_left", 0)
    acc_imad = ba_pairs * imad_per_pair + ba_left * imad_per_add if ba_pairs else adds * imad_per_add
    achieved = acc_imad / (acc_ms / 1e3)
    roofline = {"bound": "int32", "kernel": "msm_accumulate_kernel<G1>", "achieved": achieved / 1e12,
                "peak": hw_peak / 1e12, "unit": "TIMAD/s", "frac": achieved / hw_peak, "traffic": None,
                "algorithmic": (f"{ba_pairs} batch-affine pair additions x {imad_per_pair} IMAD (5 products x 256 + 1 squaring x 200) "
                                f"+ {ba_left} remaining elements x {imad_per_add} IMAD (mixed XYZZ: 6 products x 256, 2 squarings "
                                f"x 200, Y3's two products sharing a reduction 384), {adds} keys in all"
                                if ba_pairs else
                                f"{adds} mixed additions x {imad_per_add} IMAD (6 products x 256, 2 squarings x 200, "
                                f"Y3's two products sharing a reduction 384) per launch"),
                "kernels": ("ba_pass_a/ba_pass_b x 3 rounds + product-tree batch inversions + msm_accumulate_kernel<G1, direct>"
                            if ba_pairs else "msm_accumulate_kernel<G1>"),
                "peak_source": (f"zk_probe_int_pipe, measured in this run: the hardware issue rate of plain mad.lo.u32 "
                                f"({pipe['mad_lo_per_clk_sm']:.1f}/clk/SM x {pipe['num_sms']} SMs x {pipe['sm_clock_ghz']:.3f} GHz "
                                f"measured by the probe); every one of the counted IMAD is a mad.lo or mad.hi half of a product"),
                "pipe_rates": {"mad_lo_per_clk_sm": pipe["mad_lo_per_clk_sm"], "mad_hi_per_clk_sm": pipe["mad_hi_per_clk_sm"],
                               "mad_lo_hi_pair_per_clk_sm": pipe["mad_pair_per_clk_sm"], "sm_clock_ghz": pipe["sm_clock_ghz"]},
                "frac_vs_lo_hi_pairs": achieved / pipe["mad_pair_per_s"],
                "frac_vs_own_multiply": achieved / imad,
                "own_multiply_timad": imad / 1e12,
                "msm_whole_frac_ref_ops": 256 * msm_ref_ops(n) / (stats[-1]["total_device_ms"] / 1e3) / hw_peak}
    prof = os.path.join(ROOT, "profiles", "msm_batch_affine_g1_traffic.json" if ba_pairs else "msm_accumulate_g1_traffic.json")
    if os.path.exists(prof):
        # DRAM bytes per key of the accumulation phase from one ncu capture of
        # its kernels at a smaller size, scaled by this launch's keys (the
        # capture's points exceed L2 too)
        try:
            tr = json.load(open(prof))
            roofline["traffic"] = tr["bytes_per_addition"] * adds
            roofline["traffic_source"] = (f"ncu dram__bytes_read+write of the accumulation kernels at 2^{tr['capture_log_n']} "
                                          f"({tr['bytes_per_addition']:.1f} B per key) x {adds} keys")
        except (OSError, ValueError, KeyError):
            pass

    # e2e: host buffers (pinned), copies inside the timed region
    e2e = None
    if not args.no_e2e:
        pts_h = torch.empty((n, 8), dtype=torch.int64, pin_memory=True)
        sc_h = torch.empty((n, 4), dtype=torch.int64, pin_memory=True)
        pts_h.copy_(pts_d)
        sc_h.copy_(sc_d)
        pts_np = pts_h.numpy().view(np.uint64)
        sc_np = sc_h.numpy().view(np.uint64)

        def step_host():
            part = Z.msm_g1(pts_np, sc_np, device=local)
            if world > 1:
                part = D.combine(D.gather_partials(part, device=dev), Z.g1_add_affine)
            return part

        for _ in range(max(1, args.warmup // 2)):
            step_host()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step_host()
        torch.cuda.synchronize()
        dt = reduce_max((time.perf_counter() - t0) / args.steps)
        e2e = {"value": world * n / dt, "unit": "points/s", "h2d_bytes_per_step": n * (64 + 32),
               "d2h_bytes_per_step": 64 + 4 + stats[-1]["num_windows"] * 128, "ms_per_step": dt * 1e3,
               "api": "zk_msm_g1_host (pinned host points + scalars)"}

    ntt = None
    if rank == 0 and not args.no_ntt:
        ln = args.ntt_log_n
        nn = 1 << ln
        x = Z.to_device(Z.random_fr(nn, 0xA0A0 + ln), dev)
        y = torch.empty_like(x)
        for _ in range(2):
            Z.ntt(x, ln, False, out=y)
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        reps = 5
        e0.record()
        for _ in range(reps):
            Z.ntt(x, ln, False, out=y)
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / reps / 1e3
        alg_bytes = 128 * nn            # two read+write passes of 32-B elements (four-step minimum)
        alg_imad = (nn // 2) * ln * 256  # radix-2 butterflies x 256 IMAD per Montgomery multiply
        ntt = {"log_n": ln, "ms": t * 1e3, "elements_per_s": nn / t,
               "hbm": {"achieved_gbs": alg_bytes / t / 1e9, "peak_gbs": args.hbm_peak,
                       "frac": alg_bytes / t / 1e9 / args.hbm_peak, "algorithmic": "128 B per element"},
               "int32": {"achieved_timad": alg_imad / t / 1e12, "peak_timad": hw_peak / 1e12, "frac": alg_imad / t / hw_peak,
                         "frac_vs_own_multiply": alg_imad / t / imad,
                         "algorithmic": "(n/2) log2 n Montgomery multiplications x 256 IMAD, against the mad.lo issue rate"}}
        del x, y
        # the reference-shaped entry point zk_ntt (synchronous, device pointers: the
        # call bn254::ntt_gpu makes), wall time per call at config 3's sizes; the
        # reference arm times the reference's own ntt_gpu the same way on this GPU
        ntt["zk_ntt_wall_ms"] = {}
        for lr in (16, 20, 24):
            xr = Z.to_device(Z.random_fr(1 << lr, 0xA1A1 + lr), dev)
            yr = torch.empty_like(xr)
            Z.ntt_ref(yr, xr, lr, False)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(3):
                Z.ntt_ref(yr, xr, lr, False)
            torch.cuda.synchronize()
            ntt["zk_ntt_wall_ms"][f"2^{lr}"] = 1e3 * (time.perf_counter() - t0) / 3
            del xr, yr

    prove = None
    if not args.no_prove and (rank == 0 or world > 1):
        prove = bench_prove(Z, args, dev, world, rank)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import pyoracle as O
        m = 1 << args.cpu_log_n
        ph = Z.to_host(pts_d[:m])
        sh = sc[:m]
        cores = os.cpu_count() or 1
        t0 = time.perf_counter()
        O.msm_g1(ph, sh, nthreads=cores)
        dt = time.perf_counter() - t0
        cpu = {"value": m / dt, "unit": "points/s", "cores": cores, "kind": "port", "host": host_cpu(),
               "sample": f"first 2^{args.cpu_log_n} of the rank-0 points/scalars, oracle Pippenger "
                         f"(reference windows c={'/'.join(map(str, (14 if m <= 1 << 18 else 15,)))}), {cores} threads"}

    if rank == 0:
        emit({"metric": METRIC, "value": value, "unit": "points/s", "n_gpus": world, "steps": args.steps,
              "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
              "vs_baseline": None, "dtype": "u32", "data": "synthetic",
              "config": {"workload": f"G1 MSM, 2^{args.log_n} points per GPU (configs[1]); sharded MSM of "
                                     f"{world} x 2^{args.log_n} points", "log_n": args.log_n,
                         "window_bits": stats[-1]["window_bits"], "num_windows": stats[-1]["num_windows"],
                         "parallelism": f"points sharded over {world} GPU(s), partial sums all-gathered",
                         "l2": "inputs 1.5 GiB per GPU > 126 MB L2 (no flush needed)"},
              "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "ntt": ntt, "prove": prove,
              "vs_cpu_baseline": ({"device": value / cpu["value"], "e2e": e2e["value"] / cpu["value"] if e2e else None}
                                  if cpu else None),
              "clocks": sampler.summary(), "accumulate_ms": acc_ms,
              "phase_ms": {k: round(v, 3) for k, v in stats[-1]["phase_ms"].items()}})
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--log-n", type=int, default=24)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-log-n", type=int, default=18)
    ap.add_argument("--ref-sample", type=int, default=1 << 18)
    ap.add_argument("--no-ntt", action="store_true")
    ap.add_argument("--no-prove", action="store_true")
    ap.add_argument("--no-cold", action="store_true", help="skip the ZKMLPK3 cold-start measurement")
    ap.add_argument("--prove-channels", type=int, default=32)
    ap.add_argument("--prove-hw", type=int, default=32)
    ap.add_argument("--prove-steps", type=int, default=3)
    ap.add_argument("--ntt-log-n", type=int, default=24)
    ap.add_argument("--hbm-peak", type=float, default=None, help="HBM GB/s (default: MEASURED_PEAKS.json)")
    args = ap.parse_args()
    if args.hbm_peak is None:
        try:
            args.hbm_peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"])
        except (OSError, ValueError, KeyError):
            args.hbm_peak = 6650.0  # fallback measurement of this pool
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
