"""The per-rank work of zkml_dist.sharded_prove done by the CPU oracle
(oracle/groth16_oracle.py), so that the split of a proof over ranks can be
checked on CPU with gloo ranks.  Test infrastructure only."""
import numpy as np
import torch

import groth16_oracle as G
import pyoracle as O

_KEYS = {"a": "A", "b2": "B2", "l": "L", "h": "H", "b1": "B1"}


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint64).view(np.int64).copy())


def _np(t):
    return t.detach().cpu().numpy().view(np.uint64)


class OracleProver:
    def __init__(self, pk, mats):
        self.pk, self.mats = pk, mats
        self.n, self.log_n, self.m = pk["n"], pk["log_n"], pk["m"]
        self.num_public, self.l, self.n_h = pk["num_public"], pk["l"], pk["n"]
        self.g = O.fr_from_int(G.coset_shift(self.log_n))
        self.zinv = pow((pow(G.coset_shift(self.log_n), self.n, G.R) - 1) % G.R, -1, G.R)

    def error(self, msg):
        return RuntimeError(msg)

    def sync_time(self):
        import time
        return time.perf_counter()

    def timer(self):
        import time
        return time.perf_counter()

    def elapsed(self, start):
        import time
        dt = time.perf_counter() - start
        return lambda: dt

    def upload_witness(self, witness):
        return _t(witness)

    def matvec_rows(self, w, lo, hi):
        w_int = [O.fr_to_int(x) for x in _np(w)]
        out = np.zeros((3, hi - lo, 4), np.uint64)
        for k, e in enumerate(self.mats):
            full = G.matvec(e, w_int, self.n, self.m)
            for i in range(lo, hi):
                out[k, i - lo] = O.fr_from_int(full[i])
        return _t(out)

    def check_rows(self, abc, row0):
        a, b, c = (_np(abc[k]) for k in range(3))
        for i in range(a.shape[0]):
            if O.fr_to_int(a[i]) * O.fr_to_int(b[i]) % G.R != O.fr_to_int(c[i]):
                return row0 + i
        return -1

    def pad_rows(self, v, rows):
        if v.shape[0] == rows:
            return v
        out = torch.zeros((rows, 4), dtype=v.dtype)
        out[:v.shape[0]] = v
        return out

    def empty_vector(self):
        return torch.zeros((self.n, 4), dtype=torch.int64)

    def to_coset(self, v):
        coeffs = O.ntt(_np(v), self.log_n, True)
        return _t(O.coset_ntt(coeffs, self.log_n, False, self.g))

    def h_from_cosets(self, a, b, c):
        a, b, c = _np(a), _np(b), _np(c)
        q = np.stack([O.fr_from_int((O.fr_to_int(a[i]) * O.fr_to_int(b[i]) - O.fr_to_int(c[i])) * self.zinv % G.R)
                      for i in range(self.n)])
        return _t(O.coset_ntt(q, self.log_n, True, self.g))

    def stack(self, vs):
        return torch.stack(list(vs))

    def local_ntt(self, v, log_m, inverse):
        v.copy_(_t(O.ntt(_np(v), log_m, inverse)))

    def cross(self, v, log_n, s_log, part, inverse, mode, factor, factor_inverse):
        """The cross-part step of a split transform as its defining sums
        (zkml_dist.split_compute_h): the N-point DFT over the parts, written
        directly, with the twiddles w^(j1 k2) / w^(j2 k1) and the factor."""
        R = G.R
        N, n = 1 << s_log, 1 << log_n
        m = n >> s_log
        q = m >> s_log
        w = O.fr_to_int(O.compute_omega(log_n, inverse))
        wN = pow(w, m, R)
        x = [O.fr_to_int(e) for e in _np(v)]
        g = O.fr_to_int(factor) if factor is not None else None
        if g is not None and factor_inverse:
            g = pow(g, -1, R)
        ninv = pow(N, -1, R) if inverse else 1
        out = [0] * m
        for vv in range(q):
            j = part * q + vv
            xs = []
            for a in range(N):
                t = x[a * q + vv]
                if mode == 0:
                    t = t * pow(w, a * j, R) % R
                elif g is not None:
                    t = t * pow(g, a * m + j, R) % R
                xs.append(t)
            for k in range(N):
                y = sum(xs[a] * pow(wN, a * k, R) for a in range(N)) % R
                if mode == 0:
                    if g is not None:
                        y = y * pow(g, k * m + j, R) % R
                else:
                    y = y * pow(w, j * k, R) % R
                out[k * q + vv] = y * ninv % R
        return _t(np.stack([O.fr_from_int(y) for y in out]))

    def pointwise(self, a, b, c):
        a, b, c = _np(a), _np(b), _np(c)
        return _t(np.stack([O.fr_from_int((O.fr_to_int(a[i]) * O.fr_to_int(b[i]) - O.fr_to_int(c[i])) * self.zinv % G.R)
                            for i in range(a.shape[0])]))

    def h_msm_blocks(self, h_part, s_log, part):
        N = 1 << s_log
        m = self.n >> s_log
        q = m >> s_log
        idx = [k * m + part * q + v for k in range(N) for v in range(q)]
        sc = _np(h_part)
        keep = [i for i, g in enumerate(idx) if g < self.n_h]
        if not keep:
            return np.zeros(8, np.uint64)
        pts = np.stack([self.pk["H"][idx[i]] for i in keep])
        return O.msm_g1(pts, sc[keep])

    def msm(self, key, lo, hi, scalars, off):
        pts = self.pk[_KEYS[key]][lo:hi]
        words = 16 if key == "b2" else 8
        if hi <= lo:
            return np.zeros(words, np.uint64)
        sc = _np(scalars)[off + lo:off + hi]
        return O.msm_g2(pts, sc) if key == "b2" else O.msm_g1(pts, sc)

    def witness_msms(self, w, lo, hi):
        """A, B2, B1 over the witness slice [lo, hi), L over its private part."""
        import zkml_dist as D
        pub = self.num_public
        num_priv = max(0, min(self.l, self.m - 1 - pub))
        sums = {"a": self.msm("a", lo, hi, w, 0), "b2": self.msm("b2", lo, hi, w, 0), "b1": self.msm("b1", lo, hi, w, 0),
                "h": np.zeros(8, np.uint64)}
        l_lo, l_hi = max(lo, 1 + pub), min(hi, 1 + pub + num_priv)
        sums["l"] = self.msm("l", l_lo - 1 - pub, l_hi - 1 - pub, w, 1 + pub) if l_hi > l_lo else np.zeros(8, np.uint64)
        return D.pack_sums(sums)

    def start_witness_msms(self, w, lo, hi, overlap=True):
        rec = self.witness_msms(w, lo, hi)
        return lambda: (rec, lambda: 0.0)

    def add_g1(self, a, b):
        one = O.fr_from_int(1)
        return O.msm_g1_naive(np.stack([a, b]), np.stack([one, one]))

    def add_g2(self, a, b):
        one = O.fr_from_int(1)
        return O.msm_g2_naive(np.stack([a, b]), np.stack([one, one]))

    def assemble_parts(self, r, s, parts):
        import zkml_dist as D
        tot = {}
        for k in D.MSM_ORDER:
            add = self.add_g2 if k == "b2" else self.add_g1
            tot[k] = D.combine([D.unpack_sums(p)[k] for p in parts], add)
        return self.assemble(r, s, D.pack_sums(tot))

    def assemble(self, r, s, sums):
        q = np.asarray(sums, dtype=np.uint64)
        return G.assemble(self.pk, q[0:8], q[8:24], q[24:32], q[32:40], q[40:48], r, s)
