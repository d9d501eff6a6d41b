/*
 * zkml_b200.h -- C ABI of the B200 (sm_100a) Groth16 proving hot path:
 * BN254 Pippenger MSM over G1 and G2, and the Fr NTT / INTT / coset NTT.
 *
 * Drop-in boundary for gdtsitlauri/cuda-zkml.  The first group of entry
 * points mirrors the reference's C++ functions one for one (same argument
 * meaning, host/device placement and struct layouts); the reference links to
 * them through the thin C++ layer in cuda-zkml_b200/csrc/compat.cpp, which
 * exports the exact bn254:: signatures.  The second group is the B200-native
 * interface: packed device-resident data, an explicit device and CUDA stream,
 * and status codes instead of exit().
 *
 * Data layouts (all little-endian, Montgomery form, R = 2^256):
 *   Fr, Fp              32 B   4 x uint64 limbs (src/field/fp.cuh:30-34, :322-323)
 *   ref G1 affine       72 B   x(32) y(32) bool infinity at byte 64 + 7 pad
 *                              (bn254::G1Affine, src/curve/g1.cuh:29-38)
 *   ref G2 affine      136 B   x.c0 x.c1 y.c0 y.c1 (4 x 32) bool at byte 128
 *                              (bn254::G2Affine, src/curve/g2.cuh:25-33)
 *   ref G1 Jacobian     96 B   X Y Z (src/curve/g1.cuh:59-61)
 *   ref G2 Jacobian    192 B   X Y Z over Fp2 (src/curve/g2.cuh:89-91)
 *   packed G1 affine    64 B   x y; the all-zero record is the point at infinity
 *   packed G2 affine   128 B   x.c0 x.c1 y.c0 y.c1; all-zero is infinity
 *
 * Every entry point returns ZK_OK or a ZK_ERR_* code; zk_last_error() gives a
 * thread-local message.  Nothing in this library falls back to the CPU: on a
 * machine without a usable CUDA device every compute call fails with
 * ZK_ERR_NODEV.
 */
#ifndef ZKML_B200_H
#define ZKML_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZK_OK 0
#define ZK_ERR_INVALID 1  /* bad argument: null pointer, negative size, log_n out of range */
#define ZK_ERR_CUDA 2     /* CUDA runtime error */
#define ZK_ERR_NOMEM 3    /* device or pinned-host allocation failed */
#define ZK_ERR_NODEV 4    /* no usable CUDA device */
#define ZK_ERR_RANGE 5    /* size beyond what the entry point supports */

#define ZK_NTT_MAX_LOG 28      /* 2-adicity of BN254 r */
#define ZK_REF_NTT_MAX_LOG 24  /* the reference's limit, gpu_config::NTT_MAX_LOG (src/common.cuh:78) */

/* Thread-local description of the last error (empty string after success). */
const char* zk_last_error(void);
/* Number of CUDA devices visible to this process (0 when none). */
int zk_device_count(int* count);
/* Library version, major * 10000 + minor * 100 + patch. */
int zk_version(void);

/* ==================================================================
 * Reference-shaped entry points.  Synchronous; they run on the calling
 * thread's current CUDA device and its legacy default stream, as the
 * reference does.
 * ================================================================== */

/* Replaces bn254::msm_g1(const G1Affine* h_points, const Fr* h_scalars, int n)
 * (src/msm/msm.cuh:67, src/msm/msm.cu:320-442).  h_points: n host ref-G1
 * records (72 B); h_scalars: n host Fr (Montgomery).  Writes the sum as a
 * ref G1 Jacobian (96 B): (x, y, one) or the identity (0, one, 0). */
int zk_msm_g1(const void* h_points, const void* h_scalars, int n, void* out_jacobian);

/* Replaces bn254::msm_g2(const G2Affine*, const Fr*, int) (src/msm/msm.cuh:68,
 * src/msm/msm.cu:526-598).  ref G2 records (136 B) in, ref G2 Jacobian (192 B)
 * out. */
int zk_msm_g2(const void* h_points, const void* h_scalars, int n, void* out_jacobian);

/* Replaces bn254::ntt_gpu(Fr* d_out, const Fr* d_in, int log_n, bool inverse)
 * (src/ntt/ntt.cuh:49, src/ntt/ntt.cu:354-465): natural order in and out,
 * inverse scaled by n^-1, device pointers, d_out may equal d_in.  log_n above
 * ZK_REF_NTT_MAX_LOG returns ZK_ERR_RANGE with the output untouched (the
 * reference prints and returns, ntt.cu:357-361). */
int zk_ntt(void* d_out, const void* d_in, int log_n, int inverse);

/* Replaces bn254::ntt_gpu_inplace(Fr* d_data, int log_n, bool inverse)
 * (src/ntt/ntt.cuh:50, src/ntt/ntt.cu:467-478). */
int zk_ntt_inplace(void* d_data, int log_n, int inverse);

/* Replaces bn254::compute_omega / compute_omega_inv (src/ntt/ntt.cuh:53-54,
 * src/ntt/ntt.cu:64-106): the primitive 2^log_n-th root of unity (or its
 * inverse) as a Montgomery Fr, 0 <= log_n <= 28. */
int zk_compute_omega(int log_n, int inverse, void* out_fr);

/* ==================================================================
 * B200-native entry points.  `stream` is a cudaStream_t (NULL = the CUDA
 * legacy default stream, as in the CUDA runtime API).  Calls are ordered on
 * that stream; those that return a point to the host synchronise it before
 * returning.
 * ================================================================== */

/* G1 MSM over device-resident packed points (64 B) and Fr scalars.
 * out_affine: 64 host bytes (x, y Montgomery; all-zero for the identity). */
int zk_msm_g1_device(int device, void* stream, const void* d_points, const void* d_scalars,
                     size_t n, void* out_affine);
/* G1 MSM from HOST packed points and scalars: the copies to the device are
 * pipelined with the scalar decomposition and bucket sort. */
int zk_msm_g1_host(int device, void* stream, const void* h_points, const void* h_scalars,
                   size_t n, void* out_affine);
/* G2 MSM over device-resident packed points (128 B); out_affine: 128 host bytes. */
int zk_msm_g2_device(int device, void* stream, const void* d_points, const void* d_scalars,
                     size_t n, void* out_affine);
int zk_msm_g2_host(int device, void* stream, const void* h_points, const void* h_scalars,
                   size_t n, void* out_affine);

/* NTT over device memory.  inverse: 0 forward (omega), 1 inverse (omega^-1,
 * scaled by n^-1).  coset_shift: NULL for the plain transform, else a host
 * Montgomery Fr g giving
 *   forward : out = NTT(a_i * g^i)
 *   inverse : out_i = INTT(a)_i * g^-i
 * which are the coset evaluations and interpolations of compute_h
 * (src/prover/groth16.cu:350-383).  0 <= log_n <= ZK_NTT_MAX_LOG. */
int zk_ntt_device(int device, void* stream, void* d_out, const void* d_in, int log_n,
                  int inverse, const void* coset_shift);

/* Allocation-free NTT.  No counterpart in the reference: it is an addition for
 * callers that must not allocate device memory when they transform, such as a
 * latency-critical pipeline that cannot tolerate cudaMalloc / cudaFree (which
 * may synchronise the whole device and stall every stream), or a process
 * whose device memory is all reserved by its own pool allocator.
 *
 * Same arguments and bit-identical results as zk_ntt_device, for
 * 0 <= log_n <= ZK_NTT_NOALLOC_MAX_LOG (2^18 elements); a larger log_n returns
 * ZK_ERR_RANGE and launches nothing.  The call allocates nothing, on the
 * device or through any library: its working buffer (8 MiB) and its twiddle
 * and coset tables (128 KiB) live in one fixed array compiled into this
 * library, one per device.
 *  - The first call on each device does one-time set-up (it looks up that
 *    array's device address and loads the kernels it launches).  Make that
 *    first call before any stream capture begins.
 *  - Every call on a device uses the same array.  Calls whose work can
 *    overlap in time (different streams, or different host threads without a
 *    synchronisation between them) race and corrupt each other's results:
 *    issue them in order on one stream.
 *  - Nothing in the array has to start at zero: each call writes its tables
 *    and its buffer before reading them.
 *  - Asynchronous on `stream` like zk_ntt_device (NULL: legacy default
 *    stream); d_out may equal d_in. */
#define ZK_NTT_NOALLOC_MAX_LOG 18
int zk_ntt_device_noalloc(int device, void* stream, void* d_out, const void* d_in, int log_n,
                          int inverse, const void* coset_shift);

/* Quotient polynomial of compute_h after the sparse matvec
 * (src/prover/groth16.cu:322-383): from the evaluation vectors A*w, B*w, C*w
 * on the size-2^log_n domain, writes the n coefficients of
 * h = (A B - C) / (x^n - 1) to d_h, using the coset g = 5 (7 when 5^n = 1).
 * All buffers are device memory; d_h may alias d_a. */
int zk_compute_h_device(int device, void* stream, void* d_h, const void* d_a, const void* d_b,
                        const void* d_c, int log_n);

/* out_i = k_i * G for the curve generator G (G1: 64-B packed records; G2:
 * 128-B), k_i Montgomery Fr, all in device memory.  Used to generate proving
 * keys and synthetic inputs on the device. */
int zk_g1_fixed_base_device(int device, void* stream, void* d_out, const void* d_scalars, size_t n);
int zk_g2_fixed_base_device(int device, void* stream, void* d_out, const void* d_scalars, size_t n);

/* Host-side point helpers on packed affine records (used to combine the
 * per-GPU partial results of a sharded MSM). */
int zk_g1_add_affine(const void* a, const void* b, void* out);
int zk_g2_add_affine(const void* a, const void* b, void* out);

/* Measured throughput of the INT32 multiply-add pipe on `device` in IMAD per
 * second: the library's own Montgomery multiplication timed on independent
 * chains at full occupancy, 256 IMAD per multiplication.  The denominator of
 * the MSM and NTT rooflines. */
int zk_probe_imad_rate(int device, double* imad_per_second);

/* Hardware issue rate of the 32-bit integer multiply-add on `device`, measured
 * with no field code: independent chains of one instruction form at full
 * occupancy.  mad_lo: mad.lo.u32; mad_hi: mad.hi.u32; mad_pair: the two halves
 * of one 32 x 32-bit product with carry (mad.lo.cc.u32 + madc.hi.u32, counted
 * as 2 instructions), the form every Montgomery product here is made of.  The
 * per-clock figures use the SM clock the probe itself measured (clock64 over
 * the global timer).  The hardware denominators of the MSM and NTT rooflines. */
typedef struct {
    double mad_lo_per_s, mad_hi_per_s, mad_pair_per_s;
    double sm_clock_ghz;
    double mad_lo_per_clk_sm, mad_hi_per_clk_sm, mad_pair_per_clk_sm;
    int num_sms;
} zk_int_pipe_rates;
int zk_probe_int_pipe(int device, zk_int_pipe_rates* out);

/* Statistics of the most recent MSM on the calling thread: launches of this
 * library's kernels and the device time of the bucket-accumulation kernel. */
typedef struct {
    int kernel_launches;   /* kernels of this library launched by the call */
    float accumulate_ms;   /* device time of the bucket-accumulation kernel */
    float total_device_ms; /* device time from the first copy/launch to the last */
    int window_bits;       /* c */
    int num_windows;       /* W */
    long long bucket_adds; /* nonzero signed digits = mixed additions performed */
    /* device time per phase: count, scan, scatter, accumulate, fixup, reduce,
     * window sums, result copy */
    float phase_ms[8];
    /* G1 MSMs with enough keys per bucket first add each bucket's points in
     * affine pairs sharing one inversion per round: the pair additions made,
     * and the elements left for the mixed XYZZ accumulation (0 when unused) */
    long long batch_affine_pairs;
    long long batch_affine_left;
} zk_msm_stats;
int zk_msm_last_stats(zk_msm_stats* out);

/* ==================================================================
 * Groth16 prover (device-resident proving key and constraint system)
 * ================================================================== */
typedef struct zk_r1cs zk_r1cs;              /* constraint system in device CSR form */
typedef struct zk_groth16_pk zk_groth16_pk;  /* proving key resident on one device */

/* Upload an R1CS given as the reference's zkml::R1CS triplet vectors
 * (SparseEntry {int32 row; int32 col; Fr value}, 40 B; src/prover/circuit.cuh:
 * 31-49).  The evaluation domain is QAP::from_r1cs's: the next power of two
 * >= num_constraints, at least 4 (src/prover/groth16.cu:225-242); entries
 * outside the domain or the witness are ignored, as compute_h does
 * (groth16.cu:278-292). */
int zk_r1cs_create(int device, int num_constraints, int num_variables, int num_public,
                   const void* a_entries, size_t a_nnz, const void* b_entries, size_t b_nnz,
                   const void* c_entries, size_t c_nnz, zk_r1cs** out);
void zk_r1cs_destroy(zk_r1cs* r1cs);
int zk_r1cs_domain(const zk_r1cs* r1cs, int* log_n);

/* Trusted setup on the device for the given toxic waste (5 Montgomery Fr:
 * tau, alpha, beta, gamma, delta; the reference draws them in this order,
 * groth16.cu:468-472): QAP evaluations at tau on the host, every query point
 * k * G by the fixed-base kernel.  Replaces Groth16Prover::setup's point loop
 * (groth16.cu:446-642); the key is byte-identical for the same toxic waste. */
int zk_groth16_setup(zk_r1cs* r1cs, const void* toxic, zk_groth16_pk** out);
/* ZKMLPK3 proving-key files (ProvingKey::save / load_streaming,
 * groth16.cu:1104-1314), loaded straight into device memory: pieces of whole
 * records read by several threads into pinned staging, copied and converted on
 * the GPU while the next piece is read.  The first load of the process pins
 * 3 x 32 MiB of host staging (less for a smaller key; ZKML_PK_LOAD_CHUNK_MB
 * sets the piece size) and keeps it for later loads until the process exits. */
int zk_groth16_pk_load(int device, const char* path, zk_groth16_pk** out);
/* The calling thread's last zk_groth16_pk_load: bytes of query records read,
 * host time spent reading them (parallel reads into pinned chunks, overlapped
 * with the copies to the device), the whole call up to the release of its
 * pinned staging, and the time spent allocating the device buffers and the
 * pinned staging. */
typedef struct {
    double bytes;
    double read_ms;
    double total_ms;
    double alloc_ms;
} zk_pk_load_stats;
int zk_groth16_pk_last_load_stats(zk_pk_load_stats* out);
int zk_groth16_pk_save(const zk_groth16_pk* pk, const char* path);
/* vk.bin (save_vk, src/verifier/verifier.cu:103-148); keys from setup only. */
int zk_groth16_vk_save(const zk_groth16_pk* pk, const char* path);
/* Copy the verification-key points (packed affine, Montgomery); returns the
 * number of IC points and copies at most ic_capacity of them. */
int zk_groth16_vk_points(const zk_groth16_pk* pk, void* alpha1, void* beta2, void* gamma2,
                         void* delta2, void* ic, int ic_capacity);
void zk_groth16_pk_destroy(zk_groth16_pk* pk);

/* Groth16Prover::prove (groth16.cu:655-920) with the key and circuit resident:
 * h_witness = Fr[num_variables] on the host, r and s the blinding scalars
 * (Montgomery Fr; the reference draws them with mt19937_64, seed 0xCAFEBABE
 * under ZKML_DETERMINISTIC_PROVE=1, groth16.cu:709-715).  Writes the 256-byte
 * proof (Groth16Proof::serialize, groth16.cu:1058-1074) and, if `points` is
 * not NULL, A (64 B) | B (128 B) | C (64 B) packed affine. */
int zk_groth16_prove(zk_groth16_pk* pk, const zk_r1cs* r1cs, void* stream, const void* h_witness,
                     const void* r, const void* s, void* proof256, void* points);

typedef struct {
    float matvec_ms;     /* witness copy + sparse A*w, B*w, C*w */
    float compute_h_ms;  /* 7 NTTs with the fused coset steps */
    float msm_ms[5];     /* A, B (G2), L, H, B1: H from its start, the other four (run side by side) from the end of their shared sort */
    float total_ms;      /* whole prove, device time incl. host assembly */
} zk_prove_stats;
int zk_groth16_last_stats(zk_prove_stats* out);

/* ------------------------------------------------------------------
 * Pieces of zk_groth16_prove for a prove split across devices (one process
 * per GPU).  The reference proves on device 0 only; these entry points let a
 * host driver shard every step and get the same proof bytes:
 *   rows of the matvec and the witness check -> A w, B w, C w re-laid out
 *   cyclically over the parts -> each transform of compute_h split over the
 *   parts (zk_ntt_device on the part's share + one all-to-all +
 *   zk_ntt_cross_device) -> zk_compute_h_pointwise_device on each part ->
 *   the H MSM over each part's coefficients (zk_groth16_h_msm_blocks_device)
 *   and the witness MSMs over witness slices -> fold the partial sums ->
 *   zk_groth16_assemble.  (Part counts that are not powers of two: each
 *   polynomial's INTT + coset NTT on one part, then broadcasts.)
 * zk_groth16_prove runs the witness check too: unless ZKML_SKIP_WITNESS_CHECK
 * is "1" it fails with ZK_ERR_INVALID naming the first constraint whose
 * (A w)(B w) != (C w), like Groth16Prover::prove (groth16.cu:691-697) with
 * R1CS::verify_witness (src/prover/circuit.cuh:93-124).
 * ------------------------------------------------------------------ */

/* Rows [row_lo, row_hi) of A w, B w, C w (d_witness: device Fr[num_variables])
 * into d_out3 = three consecutive vectors of row_hi - row_lo Fr; rows at or
 * beyond num_constraints are zero.  row_hi <= the domain size. */
int zk_r1cs_matvec_rows_device(const zk_r1cs* r1cs, void* stream, const void* d_witness,
                               uint64_t row_lo, uint64_t row_hi, void* d_out3);
/* *first_bad = row0 + the first i < count with a_i b_i != c_i, or -1.
 * Synchronous on `stream`. */
int zk_fr_hadamard_check_device(int device, void* stream, const void* d_a, const void* d_b,
                                const void* d_c, size_t count, uint64_t row0, long long* first_bad);
/* compute_h's coset shift g (5, or 7 when 5^n = 1; groth16.cu:329-342). */
int zk_compute_h_coset_shift(int log_n, void* out_g);
/* d_out = (a b - c) / (g^n - 1) elementwise over `count` (<= 2^log_n) coset
 * evaluations of the 2^log_n-point domain (groth16.cu:364-371): all of them,
 * or one part's share; d_out may alias an input. */
int zk_compute_h_pointwise_device(int device, void* stream, void* d_out, const void* d_a,
                                  const void* d_b, const void* d_c, int log_n, uint64_t count);
/* One part's step of a 2^log_n-point (I)NTT split over 2^log_parts parts
 * (log_parts <= 3, 2 log_parts <= log_n), replacing ntt_gpu (src/ntt/ntt.cu:
 * 354-478) inside compute_h (groth16.cu:306-383) on several GPUs.  With
 * m = n / N, q = m / N, part p holds m values either "cyclic" (local t is
 * global p + N t) or in "blocks" (local k q + v is global k m + p q + v).
 * mode 0 (cyclic -> blocks, after zk_ntt_device of size m on each part's
 * cyclic values and an all-to-all sending local [p' q, p' q + q) to part p'):
 * d_in holds what the parts sent, in part order; d_out gets this part's
 * blocks of the transform, times factor(global index) if factor_g is given.
 * mode 1 (blocks -> cyclic, before the all-to-all sending local block k to
 * part k and zk_ntt_device of size m on what each part gathered): d_in holds
 * this part's blocks, times factor(global index) if given.  factor = g^i, or
 * g^-i with factor_inverse; an inverse transform's N^-1 is applied here (the
 * size-m INTT applies m^-1).  d_out must not alias d_in. */
int zk_ntt_cross_device(int device, void* stream, void* d_out, const void* d_in, int log_n, int log_parts,
                        int part, int inverse, int mode, const void* factor_g, int factor_inverse);

/* Device-resident query arrays of a proving key (packed affine, Montgomery). */
typedef struct {
    int device;
    int m;            /* entries of a, b1, b2 */
    int num_public;
    int l;            /* entries of l_query */
    int n_h;          /* entries of h_query */
    const void* a;    /* G1, 64 B each */
    const void* b1;   /* G1 */
    const void* b2;   /* G2, 128 B each */
    const void* l_query;
    const void* h_query;
} zk_groth16_arrays;
int zk_groth16_pk_arrays(const zk_groth16_pk* pk, zk_groth16_arrays* out);

/* Proof from the five MSM sums (packed affine: A 64 B | B2 128 B | L 64 B |
 * H 64 B | B1 64 B = 384 B) and the blinding scalars, as the assembly of
 * Groth16Prover::prove (groth16.cu:774-844); writes the 256-byte proof and,
 * if `points` is not NULL, A | B | C packed affine. */
int zk_groth16_assemble(const zk_groth16_pk* pk, const void* r, const void* s, const void* sums,
                        void* proof256, void* points);
/* The H MSM of a proof, sum_{i in [lo, hi)} h_i H_i over the key's H query
 * (groth16.cu:817), with d_h the n_h device coefficients of h.  From 2^16
 * points, for a slice of at least 3/4 of the query, it runs over precomputed
 * window tables of the query (2^(c j) H_i: c = 20 and 13 tables, 3.5 GB, at
 * 2^22); all windows then share one bucket set and one reduce.  Without
 * tables the plain MSM runs, and the first such call (or the end of the first
 * proof) starts building them on a stream of the key's own (about 0.55 s of
 * GPU time at 2^22); zk_groth16_precompute builds them and waits.  Smaller
 * slices run the plain MSM. */
int zk_groth16_h_msm_device(zk_groth16_pk* pk, void* stream, const void* d_h, uint64_t lo, uint64_t hi,
                            void* out_affine);
/* One part's share of the H MSM of a proof split over 2^log_parts parts:
 * sum h_i H_i over the part's coefficients in the "blocks" layout of
 * zk_ntt_cross_device (d_h_part: its n / 2^log_parts local values; global
 * indices at or beyond n_h are skipped).  The part's H points, gathered in
 * that order, and window tables over them are built on first use and kept
 * with the key (one part per key). */
int zk_groth16_h_msm_blocks_device(zk_groth16_pk* pk, void* stream, const void* d_h_part, int log_parts,
                                   int part, void* out_affine);
/* The MSMs of a proof whose scalars are the witness, over the witness slice
 * [lo, hi) (d_witness: all num_variables device Fr): sum w_i A_i, w_i B2_i and
 * w_i B1_i for i in the slice, and w_i L_{i - 1 - pub} for the private i in it,
 * with one shared counting sort.  Writes A, B2, L and B1 into a 384-byte sums
 * record (the layout of zk_groth16_assemble; H is left untouched).  Runs in
 * the key's private device context (its own scratch and lock), so a host
 * thread may run it on its own stream while another runs the transforms and
 * MSMs of the device's shared context; calls on one key run one at a time. */
int zk_groth16_witness_msms_device(zk_groth16_pk* pk, void* stream, const void* d_witness, uint64_t lo,
                                   uint64_t hi, void* sums);
/* Build the key's precomputed H-query tables now (on the key's own stream;
 * `stream` is not used) and return when they are ready; otherwise the first
 * proof starts the build as it ends and proofs run without them until it is
 * done. */
int zk_groth16_precompute(zk_groth16_pk* pk, void* stream);

/* The same from nparts partial records of 384 B (one per rank), summed first. */
int zk_groth16_assemble_parts(const zk_groth16_pk* pk, const void* r, const void* s,
                              const void* parts, int nparts, void* proof256, void* points);

/* ------------------------------------------------------------------
 * The whole prove split over several devices, in C (no counterpart in the
 * reference, which proves on device 0 only; its caller is the zkml-prove CLI,
 * src/cli/prove.cu:1286 -> Groth16Prover::prove, src/prover/groth16.cu:
 * 655-920).  Every rank holds the whole proving key and R1CS on its own
 * device and ends with the same proof bytes as zk_groth16_prove:
 *   witness slices uploaded and all-gathered -> rows of the matvec and of the
 *   witness check per rank -> compute_h with every transform split over the
 *   ranks (size-n/N transform, one all-to-all, cross-rank N-point step) -> the
 *   H MSM over each rank's coefficients, the witness MSMs over witness slices
 *   beside it -> partial sums all-gathered, folded and assembled on every rank.
 * N (the rank count) is a power of two up to 8 with N^2 <= n.  Peer data
 * always lands in the receiving device's own memory before a kernel reads it.
 * ------------------------------------------------------------------ */
typedef struct zk_comm zk_comm;  /* one rank's communicator */

/* NCCL is loaded at run time (libnccl.so.2, or $ZKML_NCCL_LIB); without it
 * these return ZK_ERR_NODEV.  One process per GPU: rank 0 makes an id
 * (128 bytes), every rank receives it out of band and joins. */
int zk_comm_unique_id(void* id128);
int zk_comm_init_rank(int device, const void* id128, int nranks, int rank, zk_comm** out);
/* One process driving ndev devices: comms[i] is rank i on devices[i]. */
int zk_comm_init_all(const int* devices, int ndev, zk_comm** comms);
/* nranks ranks as host threads sharing one device (copies on the device,
 * host barriers; no NCCL): the split prove where one GPU is at hand. */
int zk_comm_init_local(int device, int nranks, zk_comm** comms);
/* Ends the communicator's pending collectives (they fail); it cannot be used again. */
int zk_comm_abort(zk_comm* comm);
void zk_comm_destroy(zk_comm* comm);

/* This rank's part of one proof (every rank calls it with the same whole host
 * witness, r and s; each returns the proof).  pk and r1cs on the rank's
 * device.  A rank whose call lasts longer than ZKML_SPLIT_TIMEOUT_S seconds
 * (default 300) aborts its communicator and returns ZK_ERR_CUDA.  A witness
 * that does not satisfy the R1CS fails on every rank with ZK_ERR_INVALID, as
 * zk_groth16_prove does. */
int zk_groth16_prove_split(zk_groth16_pk* pk, const zk_r1cs* r1cs, zk_comm* comm, const void* h_witness, const void* r,
                           const void* s, void* proof256, void* points);

typedef struct {
    int nranks, rank;
    float witness_ms;       /* this rank's witness slice upload + the all-gather (device) */
    float matvec_ms;        /* its rows of A w, B w, C w, their check and its all-reduce */
    float compute_h_ms;     /* the split transforms, all-to-alls included */
    float all_to_all_ms;    /* the all-to-alls of compute_h (one polynomial each), summed; they overlap its transforms */
    float h_msm_ms;         /* the H MSM over its coefficients */
    float witness_msms_ms;  /* A, B2, B1, L over its witness slice (side stream, overlapped) */
    float witness_wait_ms;  /* host time spent waiting for them after the H MSM */
    float gather_ms;        /* partial sums all-gather */
    float assemble_ms;      /* fold, blinding and serialisation on the host */
    float total_ms;         /* the whole call, host wall time */
} zk_split_stats;
/* Statistics of the calling thread's last zk_groth16_prove_split. */
int zk_groth16_split_last_stats(zk_split_stats* out);

/* All ranks from one call: pks[i], r1cs[i] on comms[i]'s device (comms from
 * zk_comm_init_all or zk_comm_init_local), one host thread per rank.  A rank
 * that fails aborts every communicator; after timeout_s seconds (<= 0: 600)
 * the communicators are aborted as well.  stats: NULL or nranks records. */
int zk_groth16_prove_multi(zk_groth16_pk* const* pks, const zk_r1cs* const* r1cs, zk_comm* const* comms, int nranks,
                           const void* h_witness, const void* r, const void* s, void* proof256, void* points,
                           double timeout_s, zk_split_stats* stats);

/* ------------------------------------------------------------------
 * Verifier: the BN254 optimal ate pairing and the Groth16 check, host code
 * with the public-input MSM on a GPU.
 * ------------------------------------------------------------------ */
typedef struct zk_groth16_vk zk_groth16_vk;  /* verification key (host) */

/* vk.bin (save_vk / load_vk, src/verifier/verifier.cu:103-148). */
int zk_groth16_vk_load(const char* path, zk_groth16_vk** out);
/* The verification key of a proving key made by zk_groth16_setup. */
int zk_groth16_vk_from_pk(const zk_groth16_pk* pk, zk_groth16_vk** out);
void zk_groth16_vk_destroy(zk_groth16_vk* vk);
/* Number of public inputs the key expects (-1 for NULL). */
int zk_groth16_vk_num_public(const zk_groth16_vk* vk);

/* Replaces Groth16Verifier::verify (src/prover/groth16.cu:967-1022):
 * e(-A, B) e(alpha, beta) e(vk_x, gamma) e(C, delta) == 1 with
 * vk_x = IC[0] + sum_i x_i IC[i + 1] (x: num_public Montgomery Fr) and the
 * pairing product of verify_pairing_product (src/curve/pairing.cuh:278-282).
 * proof256: Groth16Proof::serialize bytes.  vk_x is an MSM on `device`
 * (>= 0), or summed on the host with device = -1 (the reference's loop).
 * *valid = 1 when the proof verifies, 0 otherwise (a public-input count other
 * than the key's included, as the reference returns false). */
int zk_groth16_verify(const zk_groth16_vk* vk, int device, const void* public_inputs, int num_public,
                      const void* proof256, int* valid);

/* Replaces bn254::pairing (src/curve/pairing.cuh:226-230): e(P, Q) for a packed
 * G1 point (64 B) and G2 point (128 B), written as 12 Montgomery Fp (384 B) in
 * the reference's Fp12 layout (c0.c0.c0, c0.c0.c1, c0.c1.c0, ..., c1.c2.c1;
 * Fp6 = Fp2[v]/(v^3 - (9 + u)), Fp12 = Fp6[w]/(w^2 - v)); the reduced value
 * f^((p^12 - 1)/r), equal bit for bit to the reference's. */
int zk_bn254_pairing(const void* p64, const void* q128, void* out_fp12);
/* Replaces bn254::verify_pairing_product (src/curve/pairing.cuh:278-282):
 * *holds = 1 when prod_i e(P_i, Q_i) == 1 (n packed pairs). */
int zk_bn254_pairing_check(const void* p64s, const void* q128s, int n, int* holds);

/* ==================================================================
 * Synthetic workloads (seeded, for benchmarks and tests)
 * ================================================================== */

/* An R1CS with a satisfying witness, in the reference's layout: constraint
 * matrices as zkml::SparseEntry records {int32 row; int32 col; Fr value}
 * (40 B, src/prover/circuit.cuh:31-35), witness as Fr[num_variables] ordered
 * [1, public..., private...]. */
typedef struct {
    int num_constraints;
    int num_variables;
    int num_public;
    size_t nnz[3];     /* A, B, C */
    void* entries[3];  /* malloc'd SparseEntry arrays */
    void* witness;     /* malloc'd Fr array */
} zk_synth_circuit;

/* `layers` CONV2D 3x3 (pad 1) layers of channels x height x width with
 * seeded int8 weights and biases, each output through RELU_EXACT with the
 * reference's gadgets (src/prover/gadgets.cuh:197-220: a signed range check
 * of `bits` bits whose top bit selects y = z, then y = q 2^shift + r with r
 * in `shift` bits and q in the same signed range), `out_bits` replacing
 * `bits` from the second layer on (0: same), then `dense_outputs` int8 dense
 * outputs made public through equality rows.  Public inputs, in order: the
 * dense outputs, a model tag, the input feature map (values 0..16).
 * ZK_ERR_INVALID when a value leaves its layer's range. */
int zk_synth_conv_circuit(int layers, int channels, int height, int width, int bits, int shift,
                          int out_bits, int dense_outputs, uint64_t seed, zk_synth_circuit* out);
/* A quantised MLP statement: `batch` samples of n_in -> n_hidden (LINEAR +
 * RELU_EXACT with `bits`, `shift`, the gadgets above) -> n_out (LINEAR), one
 * seeded int8 model, inputs 0..16; public: the outputs, a model tag, the
 * context when `context` (bound by ctx * ctx = ctx^2, src/prover/gadgets.cuh:
 * 152-158) and the inputs.  Batch 4 of 64 -> 32 -> 10, bits 24, shift 6 has
 * the reference statement's counts for that model: 7,762 constraints, 7,764
 * variables, 298 public.  ZK_ERR_INVALID when a value leaves its range. */
int zk_synth_mlp_circuit(int batch, int n_in, int n_hidden, int n_out, int bits, int shift, int context,
                         uint64_t seed, zk_synth_circuit* out);
void zk_synth_free(zk_synth_circuit* c);

#ifdef __cplusplus
}
#endif
#endif
