"""Independent reader of the reference's ZKMLPK3 proving-key and vk.bin files
(src/prover/groth16.cu:1104-1314, src/verifier/verifier.cu:103-148), used by
the tests to check the library's writers."""
import struct

import numpy as np

P = 21888242871839275222246405745257275088696311157297823662689037894645226208583
RINV_P = pow(1 << 256, -1, P)


def mont_p(std):
    return (std << 256) % P


def _fp(buf, off):
    return int.from_bytes(buf[off:off + 32], "little"), off + 32


def parse_pk(buf):
    off = 0
    assert buf[0:7] == b"ZKMLPK3", "magic"
    off = 8
    version, n, m, pub = struct.unpack_from("<Iiii", buf, off)
    off += 16
    assert version == 3

    def g1(off):
        inf = buf[off]
        x, off2 = _fp(buf, off + 1)
        y, off2 = _fp(buf, off2)
        return (None if inf else (x, y)), off2

    def g2(off):
        inf = buf[off]
        vals = []
        o = off + 1
        for _ in range(4):
            v, o = _fp(buf, o)
            vals.append(v)
        return (None if inf else tuple(vals)), o

    def vec(off, fn):
        (cnt,) = struct.unpack_from("<i", buf, off)
        off += 4
        assert 0 <= cnt <= (1 << 28)
        out = []
        for _ in range(cnt):
            p, off = fn(off)
            out.append(p)
        return out, off

    key = {"n": n, "m": m, "num_public": pub}
    for name in ("alpha1", "beta1", "delta1"):
        key[name], off = g1(off)
    for name in ("beta2", "gamma2", "delta2"):
        key[name], off = g2(off)
    key["tau_g1"], off = vec(off, g1)
    key["tau_g2"], off = vec(off, g2)
    key["A"], off = vec(off, g1)
    key["B1"], off = vec(off, g1)
    key["B2"], off = vec(off, g2)
    key["L"], off = vec(off, g1)
    key["H"], off = vec(off, g1)
    assert off == len(buf), "trailing bytes"
    return key


def pk_size(n_h, m, l, tau_g2=2, tau_g1=0):
    """Byte size of a ZKMLPK3 file (worked check: p160 = 294,496 bytes)."""
    return 24 + 3 * 65 + 3 * 129 + (4 + tau_g1 * 65) + (4 + tau_g2 * 129) + 2 * (4 + m * 65) + (4 + m * 129) + (4 + l * 65) + (4 + n_h * 65)


def parse_vk(buf):
    (pub,) = struct.unpack_from("<i", buf, 0)
    off = 4
    vals = []
    for _ in range(2 + 3 * 4):
        v, off = _fp(buf, off)
        vals.append(v)
    (nic,) = struct.unpack_from("<i", buf, off)
    off += 4
    ic = []
    for _ in range(nic):
        x, off = _fp(buf, off)
        y, off = _fp(buf, off)
        ic.append((x, y))
    assert off == len(buf)
    return {"num_public": pub, "alpha1": tuple(vals[0:2]), "beta2": tuple(vals[2:6]), "gamma2": tuple(vals[6:10]),
            "delta2": tuple(vals[10:14]), "ic": ic}


def std_g1(rec):
    """packed Montgomery G1 record -> (x, y) standard ints, or None for infinity."""
    rec = np.asarray(rec, dtype=np.uint64)
    if not rec.any():
        return None
    vals = [sum(int(w) << (64 * i) for i, w in enumerate(rec[k:k + 4])) * RINV_P % P for k in (0, 4)]
    return tuple(vals)


def std_g2(rec):
    rec = np.asarray(rec, dtype=np.uint64)
    if not rec.any():
        return None
    return tuple(sum(int(w) << (64 * i) for i, w in enumerate(rec[k:k + 4])) * RINV_P % P for k in (0, 4, 8, 12))
