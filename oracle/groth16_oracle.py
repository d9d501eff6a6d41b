"""CPU restatement of the reference's Groth16 setup / prove / serialise, on top
of the pinned oracle (oracle/bn254_oracle.c) — TEST INFRASTRUCTURE ONLY.

Follows src/prover/groth16.cu:
  QAP::from_r1cs                    :225-242   (n = next pow2 >= constraints, >= 4)
  compute_qap_evaluations_at_tau    :97-189
  Groth16Prover::setup              :446-642   (query scalars and points)
  Groth16Prover::compute_h          :263-390   (matvec, then orc_compute_h_from_evals)
  Groth16Prover::prove              :655-844   (A, B, C assembly)
  Groth16Proof::serialize           :1058-1074
and checks a proof with the toxic waste known: the points equal their claimed
discrete logs and A_s B_s = alpha beta + vk_x gamma + C_s delta in Fr, which
with bilinearity is the pairing equation the reference verifies
(groth16.cu:967-1022); the reference's own diagnostic does the same
(groth16.cu:840-905).

R1CS triplets are numpy structured arrays with fields row (i4), col (i4),
v (u8, 4) — the reference's SparseEntry layout.
"""
import numpy as np

import pyoracle as O

R = O.R
P = O.P
ENTRY = np.dtype([("row", "<i4"), ("col", "<i4"), ("v", "<u8", (4,))])


def domain(num_constraints):
    n, log_n = 1, 0
    while n < num_constraints:
        n <<= 1
        log_n += 1
    if n < 4:
        n, log_n = 4, 2
    return n, log_n


def _ints(a):
    return [O.fr_to_int(x) for x in a]


def matvec(entries, w_int, n, m):
    """(A w) rows as Python ints mod r (rows < n, cols < m)."""
    out = [0] * n
    vals = _ints(entries["v"])
    for (row, col), v in zip(zip(entries["row"].tolist(), entries["col"].tolist()), vals):
        if row < n and col < m:
            out[row] = (out[row] + v * w_int[col]) % R
    return out


def qap_at_tau(mats, n, log_n, m, tau):
    w = O.fr_to_int(O.compute_omega(log_n, False))
    vanish = (pow(tau, n, R) - 1) % R
    ninv = pow(n, -1, R)
    lag = []
    wj = 1
    for _ in range(n):
        lag.append(vanish * wj % R * ninv % R * pow((tau - wj) % R, -1, R) % R)
        wj = wj * w % R
    at = []
    for e in mats:
        acc = [0] * m
        vals = _ints(e["v"])
        for (row, col), v in zip(zip(e["row"].tolist(), e["col"].tolist()), vals):
            if row < n and col < m:
                acc[col] = (acc[col] + v * lag[row]) % R
        at.append(acc)
    return at, vanish


def _mont(xs):
    return np.stack([O.fr_from_int(x) for x in xs]) if xs else np.zeros((0, 4), np.uint64)


def setup(mats, num_constraints, m, num_public, toxic):
    """toxic = (tau, alpha, beta, gamma, delta) as ints. Returns the key dict."""
    tau, alpha, beta, gamma, delta = toxic
    n, log_n = domain(num_constraints)
    at, vanish = qap_at_tau(mats, n, log_n, m, tau)
    dinv, ginv = pow(delta, -1, R), pow(gamma, -1, R)
    lc = [(beta * at[0][i] + alpha * at[1][i] + at[2][i]) % R for i in range(m)]
    l = max(0, m - num_public - 1)
    Lq = [lc[i + 1 + num_public] * dinv % R for i in range(l)]
    Hq = [vanish * dinv % R * pow(tau, i, R) % R for i in range(n)]
    ic = [lc[i] * ginv % R for i in range(num_public + 1)]
    g1 = O.g1_fixed_base
    g2 = O.g2_fixed_base
    return {
        "n": n, "log_n": log_n, "m": m, "num_public": num_public, "l": l,
        "A": g1(_mont(at[0])), "B1": g1(_mont(at[1])), "B2": g2(_mont(at[1])),
        "L": g1(_mont(Lq)), "H": g1(_mont(Hq)), "IC": g1(_mont(ic)),
        "alpha1": g1(_mont([alpha]))[0], "beta1": g1(_mont([beta]))[0], "delta1": g1(_mont([delta]))[0],
        "beta2": g2(_mont([beta]))[0], "gamma2": g2(_mont([gamma]))[0], "delta2": g2(_mont([delta]))[0],
        "tau2": g2(_mont([tau]))[0],
        "_at": at, "_vanish": vanish, "_toxic": toxic,
    }


def compute_h(mats, w_int, n, log_n, m):
    a, b, c = (matvec(e, w_int, n, m) for e in mats)
    return O.compute_h_from_evals(_mont(a), _mont(b), _mont(c), log_n)


def prove(pk, mats, witness, r, s):
    """witness: (m, 4) Montgomery; r, s ints. Returns (proof bytes, A, B, C)."""
    n, log_n, m, pub = pk["n"], pk["log_n"], pk["m"], pk["num_public"]
    w_int = _ints(witness)
    h = compute_h(mats, w_int, n, log_n, m)
    a_msm = O.msm_g1(pk["A"], witness)
    b_msm = O.msm_g2(pk["B2"], witness)
    num_priv = min(pk["l"], m - 1 - pub)
    l_msm = O.msm_g1(pk["L"][:num_priv], witness[1 + pub: 1 + pub + num_priv]) if num_priv > 0 else np.zeros(8, np.uint64)
    h_msm = O.msm_g1(pk["H"][:n], h)
    b1_msm = O.msm_g1(pk["B1"], witness)
    proof, A, B, C = assemble(pk, a_msm, b_msm, l_msm, h_msm, b1_msm, r, s)
    return proof, A, B, C, h


def assemble(pk, a_msm, b_msm, l_msm, h_msm, b1_msm, r, s):
    """Proof points from the five MSM sums (groth16.cu:774-844)."""
    one, rr, ss = O.fr_from_int(1), O.fr_from_int(r), O.fr_from_int(s)
    A = O.msm_g1_naive(np.stack([pk["alpha1"], a_msm, pk["delta1"]]), np.stack([one, one, rr]))
    B = O.msm_g2_naive(np.stack([pk["beta2"], b_msm, pk["delta2"]]), np.stack([one, one, ss]))
    C = O.msm_g1_naive(np.stack([l_msm, h_msm, A, pk["beta1"], b1_msm]), np.stack([one, one, ss, rr, rr]))
    return serialize(A, B, C), A, B, C


def coset_shift(log_n):
    """compute_h's coset shift (groth16.cu:329-342): 5, or 7 when 5^n = 1; as an int."""
    n = 1 << log_n
    return 5 if pow(5, n, R) != 1 else 7


def first_failing_constraint(mats, w_int, num_constraints, n, m):
    """R1CS::verify_witness (src/prover/circuit.cuh:93-124): the first row with
    (A w)(B w) != (C w), or -1."""
    a, b, c = (matvec(e, w_int, n, m) for e in mats)
    for i in range(num_constraints):
        if a[i] * b[i] % R != c[i]:
            return i
    return -1


def serialize(A, B, C):
    out = bytearray()
    for v in (A[0:4], A[4:8], B[0:4], B[4:8], B[8:12], B[12:16], C[0:4], C[4:8]):
        out += O.fp_to_int(v).to_bytes(32, "little") if np.asarray(v).any() else bytes(32)
    return bytes(out)


def trapdoor_verify(pk, witness, r, s, h, A, B, C):
    """The Groth16 equation in the exponent with the toxic waste known."""
    tau, alpha, beta, gamma, delta = pk["_toxic"]
    at, vanish = pk["_at"], pk["_vanish"]
    m, pub = pk["m"], pk["num_public"]
    w = _ints(witness)
    Aw = sum(w[i] * at[0][i] for i in range(m)) % R
    Bw = sum(w[i] * at[1][i] for i in range(m)) % R
    A_s = (alpha + Aw + r * delta) % R
    B_s = (beta + Bw + s * delta) % R
    lc = [(beta * at[0][i] + alpha * at[1][i] + at[2][i]) % R for i in range(m)]
    priv = sum(w[i] * lc[i] for i in range(1 + pub, m)) % R
    h_tau = O.fr_to_int(O.fr_poly_eval(h, O.fr_from_int(tau)))
    C_s = ((priv + h_tau * vanish) * pow(delta, -1, R) + s * A_s + r * (beta + Bw)) % R
    vk_x = sum(w[i] * lc[i] for i in range(pub + 1)) % R * pow(gamma, -1, R) % R
    ok_eq = (A_s * B_s - alpha * beta - vk_x * gamma - C_s * delta) % R == 0
    ok_pts = (np.array_equal(O.g1_fixed_base(_mont([A_s]))[0], A)
              and np.array_equal(O.g2_fixed_base(_mont([B_s]))[0], B)
              and np.array_equal(O.g1_fixed_base(_mont([C_s]))[0], C))
    return ok_eq and ok_pts


class Mt19937_64:
    """std::mt19937_64 (via the oracle) for the reference's seeded draws."""

    def __init__(self, seed):
        self.r = O.Rng(seed)

    def nonzero_fr(self):
        # random_nonzero_fr (groth16.cu:48-58): Fr::from_uint(rng()) until nonzero
        while True:
            v = self.r.next()
            if v:
                return v


def toxic_deterministic():
    """ZKML_DETERMINISTIC_SETUP=1: seed 0xDEADBEEF42, tau alpha beta gamma delta (groth16.cu:459-472)."""
    g = Mt19937_64(0xDEADBEEF42)
    return tuple(g.nonzero_fr() for _ in range(5))


def blinding_deterministic():
    """ZKML_DETERMINISTIC_PROVE=1: seed 0xCAFEBABE, r then s (groth16.cu:709-715)."""
    g = Mt19937_64(0xCAFEBABE)
    return g.nonzero_fr(), g.nonzero_fr()
