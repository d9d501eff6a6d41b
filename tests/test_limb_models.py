"""The carry-chain arithmetic of cuda-zkml_b200/csrc/field.cuh replayed on the
CPU, instruction by instruction: mac_row (the paired CIOS row), fmul, the
shared-reduction sums fmul2sum / fmulsum<K> (K <= 4) and the dedicated squaring
fsqr_inline.  Each PTX form (mad.lo/hi[.cc], madc.lo/hi[.cc], add[c][.cc]) is
applied to 32-bit words with an explicit carry flag, and the model asserts what
the kernels rely on without checking: no carry is ever dropped (an op without
.cc, or a .cc op that ends its asm block, must not carry out), t0 is zero after
every reduction row, the word above the result is zero, and the value handed to
the final conditional subtraction is below 2m.  The results are compared with
Python integers for random and edge inputs of both BN254 moduli.  The GPU tests
check the compiled kernels themselves; this pins the bounds argued in the
comments of field.cuh."""
import random

import pytest

P = 21888242871839275222246405745257275088696311157297823662689037894645226208583
R = 21888242871839275222246405745257275088548364400416034343698204186575808495617
M32 = (1 << 32) - 1
INV = {P: 0xE4866389, R: 0xEFFFFFFF}  # -m^-1 mod 2^32, as ModP / ModR


def limbs(x):
    return [(x >> (32 * i)) & M32 for i in range(8)]


def value(ws):
    return sum(w << (32 * i) for i, w in enumerate(ws))


class Chain:
    """One asm block: a carry flag threaded through its ops."""

    def __init__(self):
        self.cf = 0

    def _put(self, t, i, s, cc, use_cf):
        s += self.cf if use_cf else 0
        t[i] = s & M32
        if cc:
            self.cf = s >> 32
        else:
            assert s >> 32 == 0, "a carry was dropped"
            self.cf = 0

    def mad_lo(self, t, i, a, b, cc=True, use_cf=False):
        self._put(t, i, t[i] + ((a * b) & M32), cc, use_cf)

    def mad_hi(self, t, i, a, b, cc=True, use_cf=False):
        self._put(t, i, t[i] + ((a * b) >> 32), cc, use_cf)

    def add(self, t, i, x, cc=True, use_cf=False):
        self._put(t, i, t[i] + x, cc, use_cf)

    def end(self):
        assert self.cf == 0, "a carry left the asm block"


def mac_row(t, a, b):
    """t[0..8] += a * b[0..7]: the ZK_ROW_PAIRED form of mac_row."""
    c = Chain()
    for j in (0, 2, 4, 6):  # even limbs: words j, j + 1
        c.mad_lo(t, j, a, b[j], use_cf=j > 0)
        c.mad_hi(t, j + 1, a, b[j], use_cf=True)
    c.add(t, 8, 0, cc=False, use_cf=True)
    c = Chain()
    for j in (1, 3, 5, 7):  # odd limbs: words j, j + 1
        c.mad_lo(t, j, a, b[j], use_cf=j > 1)
        c.mad_hi(t, j + 1, a, b[j], cc=j < 7, use_cf=True)
    c.end()


def cond_sub(t, m):
    v = value(t)
    assert v < 2 * m and v < (1 << 256)
    return v - m if v >= m else v


def cios(pairs, m):
    """fmul (one pair), fmul2sum (two), fmulsum<K> (K pairs): per limb i the rows
    a_k[i] * b_k, then q = t0 * inv and the row q * m, then a one-word shift."""
    ml = limbs(m)
    t = [0] * 9
    for i in range(8):
        for a, b in pairs:
            mac_row(t, limbs(a)[i], limbs(b))
        q = (t[0] * INV[m]) & M32
        mac_row(t, q, ml)
        assert t[0] == 0
        t = t[1:] + [0]
    assert t[8] == 0
    return cond_sub(t[:8], m)


def fsqr(a, m):
    """fsqr_inline: cross products once, doubled, plus the diagonal, then a
    separate reduction with a 10-word window over the 16 words."""
    x = limbs(a)
    T = [0] * 16
    for i in range(7):  # cross-product row i: a_i * a[i+1..7]
        c = Chain()
        for j in range(i + 1, 8):  # low halves on words i + j
            c.mad_lo(T, i + j, x[i], x[j], use_cf=j > i + 1)
        c.add(T, i + 8, 0, cc=False, use_cf=True)
        c = Chain()
        for j in range(i + 1, 8):  # high halves on words i + j + 1
            last = j == 7
            c.mad_hi(T, i + j + 1, x[i], x[j], cc=not last or i == 6, use_cf=j > i + 1)
        c.end()
    c = Chain()
    for k in range(16):  # T = 2 T
        c.add(T, k, T[k], cc=k < 15, use_cf=k > 0)
    c = Chain()
    for i in range(8):  # T += a_i^2 2^(64 i)
        c.mad_lo(T, 2 * i, x[i], x[i], use_cf=i > 0)
        c.mad_hi(T, 2 * i + 1, x[i], x[i], cc=i < 7, use_cf=True)
    assert value(T) == a * a
    ml = limbs(m)
    w = T[:9] + [0]  # t0..t8, t9
    for i in range(8):
        q = (w[0] * INV[m]) & M32
        c = Chain()
        for j in (0, 2, 4, 6):
            c.mad_lo(w, j, q, ml[j], use_cf=j > 0)
            c.mad_hi(w, j + 1, q, ml[j], use_cf=True)
        c.add(w, 8, 0, use_cf=True)
        c.add(w, 9, 0, cc=False, use_cf=True)
        c = Chain()
        for j in (1, 3, 5, 7):
            c.mad_lo(w, j, q, ml[j], use_cf=j > 1)
            c.mad_hi(w, j + 1, q, ml[j], use_cf=True)
        c.add(w, 9, 0, cc=False, use_cf=True)
        assert w[0] == 0
        w = w[1:] + [0]
        if i + 9 <= 15:
            c = Chain()
            c.add(w, 8, T[i + 9])
            w[9] = c.cf
    assert w[8] == 0 and w[9] == 0
    return cond_sub(w[:8], m)


def _inputs(m, n, seed):
    rng = random.Random(seed)
    edge = [0, 1, 2, m - 1, m - 2, (m - 1) // 2, 1 << 253, (1 << 254) - 1 if (1 << 254) - 1 < m else m - 3,
            int("ffffffff" * 7, 16), value([M32] * 7 + [0]), m // 3]
    edge = [e % m for e in edge]
    vals = edge + [rng.randrange(m) for _ in range(n)]
    # values whose limbs are all large stress the carries most
    vals += [(m - 1 - rng.randrange(1 << 40)) for _ in range(n // 4)]
    return vals


RINV = {m: pow(1 << 256, -1, m) for m in (P, R)}


@pytest.mark.parametrize("m", [P, R], ids=["p", "r"])
def test_squaring(m):
    for a in _inputs(m, 1500, 1):
        assert fsqr(a, m) == a * a * RINV[m] % m, hex(a)


@pytest.mark.parametrize("m", [P, R], ids=["p", "r"])
def test_products_and_shared_reductions(m):
    vals = _inputs(m, 400, 2)
    rng = random.Random(3)
    for a in vals:
        b = rng.choice(vals)
        assert cios([(a, b)], m) == a * b * RINV[m] % m
        # fmul2sum, and fmulsub's a b + (m - c) d
        c, d = rng.choice(vals), rng.choice(vals)
        assert cios([(a, b), (c, d)], m) == (a * b + c * d) * RINV[m] % m
        assert cios([(a, b), ((m - c) % m, d)], m) == (a * b - c * d) * RINV[m] % m
    # fmulsum<K>, K <= 4 (the matvec's row dot products), with the largest inputs
    big = [m - 1 - k for k in range(8)]
    for K in (3, 4):
        pairs = [(rng.choice(vals), rng.choice(vals)) for _ in range(K)]
        assert cios(pairs, m) == sum(a * b for a, b in pairs) * RINV[m] % m
        pairs = [(big[k], big[-1 - k]) for k in range(K)]
        assert cios(pairs, m) == sum(a * b for a, b in pairs) * RINV[m] % m


def test_model_catches_a_dropped_carry():
    """The model itself: a row whose top word cannot hold the sum must fail."""
    t = [M32] * 9
    with pytest.raises(AssertionError):
        mac_row(t, M32, [M32] * 8)
