"""zk_ntt_device_noalloc, the allocation-free NTT, against zk_ntt_device.

Called straight through the C ABI.  Each case runs the new entry point twice
in a row (the second call reuses the shared fixed array the first one wrote)
and both results must equal zk_ntt_device's bit for bit.  The file is
collected last so that it also runs after every other GPU test in a process.
"""
import ctypes

import numpy as np
import pytest

import zkml_b200 as Z

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

MAX_LOG = 18  # ZK_NTT_NOALLOC_MAX_LOG

_fn = Z.lib.zk_ntt_device_noalloc
_fn.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                ctypes.c_void_p]
_fn.restype = ctypes.c_int


def noalloc(x, log_n, inverse, coset=None, out=None):
    if out is None:
        out = torch.empty_like(x)
    g = None
    if coset is not None:
        gc = np.ascontiguousarray(coset, dtype=np.uint64)
        g = gc.ctypes.data_as(ctypes.c_void_p)
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    Z.check(_fn(x.device.index, stream, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(x.data_ptr()), log_n,
                int(inverse), g))
    return out


CASES = [(0, False, None), (1, True, None), (5, False, None), (9, True, None), (12, False, None),
         (16, True, None), (17, False, None), (MAX_LOG, False, None), (MAX_LOG, True, None),
         (0, True, 5), (3, False, 5), (10, True, 5), (14, False, 7), (MAX_LOG, True, 5), (MAX_LOG, False, 5)]


@pytest.mark.parametrize("log_n,inverse,coset", CASES)
def test_two_calls_in_a_row_match_existing_entry_point(log_n, inverse, coset):
    x = Z.to_device(Z.random_fr(1 << log_n, 0x70A0 + 2 * log_n + int(inverse)))
    g = Z.fr_from_int(coset) if coset is not None else None
    want = Z.to_host(Z.ntt(x, log_n, inverse, coset=g))
    first = noalloc(x, log_n, inverse, g)
    second = noalloc(x, log_n, inverse, g)
    assert np.array_equal(Z.to_host(first), want)
    assert np.array_equal(Z.to_host(second), want)


def test_alternating_sizes_and_directions_share_the_array():
    """Calls of different sizes and directions back to back on one stream:
    each rewrites the tables the previous one left behind."""
    xs = {ln: Z.to_device(Z.random_fr(1 << ln, 0x71B0 + ln)) for ln in (MAX_LOG, 7, 13)}
    want = {(ln, inv): Z.to_host(Z.ntt(x, ln, inv)) for ln, x in xs.items() for inv in (False, True)}
    outs = []
    for ln, inv in [(MAX_LOG, False), (7, True), (13, False), (MAX_LOG, True), (7, False), (13, True)]:
        outs.append(((ln, inv), noalloc(xs[ln], ln, inv)))
    for key, out in outs:
        assert np.array_equal(Z.to_host(out), want[key]), key


def test_in_place_and_round_trip():
    ln = 15
    x = Z.to_device(Z.random_fr(1 << ln, 0x72C0))
    want = Z.to_host(Z.ntt(x, ln, False))
    y = x.clone()
    noalloc(y, ln, False, out=y)
    assert np.array_equal(Z.to_host(y), want)
    noalloc(y, ln, True, out=y)
    assert torch.equal(y, x)


def test_size_beyond_maximum_is_rejected():
    x = torch.zeros((1 << (MAX_LOG + 1), 4), dtype=torch.int64, device="cuda")
    out = torch.empty_like(x)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = _fn(x.device.index, stream, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(x.data_ptr()), MAX_LOG + 1, 0,
             None)
    assert st == Z.ZK_ERR_RANGE
    assert "log_n = 19" in Z.last_error()
    assert _fn(x.device.index, stream, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(x.data_ptr()), -1, 0,
               None) == Z.ZK_ERR_RANGE
    assert _fn(x.device.index, stream, None, ctypes.c_void_p(x.data_ptr()), 4, 0, None) == Z.ZK_ERR_INVALID
