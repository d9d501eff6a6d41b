"""C-ABI checks that need no GPU: the library loads, exports every entry point
declared in include/zkml_b200.h and the reference's bn254:: C++ symbols, the
host-only helpers agree with the golden vectors, and compute entry points
refuse to run (no CPU fallback) when no CUDA device is visible."""
import os
import subprocess

import numpy as np
import pytest

import pyoracle as O
import zkml_b200 as Z
from conftest import GOLDEN, ROOT

# The reference's link-level interface (src/msm/msm.cuh:67-68, src/ntt/ntt.cuh:49-54)
REF_SYMBOLS = [
    "bn254::msm_g1(bn254::G1Affine const*, bn254::Fr const*, int)",
    "bn254::msm_g2(bn254::G2Affine const*, bn254::Fr const*, int)",
    "bn254::ntt_gpu(bn254::Fr*, bn254::Fr const*, int, bool)",
    "bn254::ntt_gpu_inplace(bn254::Fr*, int, bool)",
    "bn254::compute_omega(int)",
    "bn254::compute_omega_inv(int)",
]


def test_exports_every_declared_symbol():
    names = Z.declared_symbols()
    assert len(names) >= 20
    for name in names:
        assert hasattr(Z.lib, name), name


def test_exports_reference_cpp_symbols():
    out = subprocess.run(["nm", "-DC", "--defined-only", Z.LIB_PATH], capture_output=True, text=True, check=True).stdout
    for sym in REF_SYMBOLS:
        assert sym in out, sym


def test_compute_omega_matches_reference():
    g = np.load(os.path.join(GOLDEN, "omega.npz"))
    for ln in range(29):
        assert np.array_equal(Z.compute_omega(ln, False), g["fwd"][ln])
        assert np.array_equal(Z.compute_omega(ln, True), g["inv"][ln])
    with pytest.raises(Z.ZkError):
        Z.compute_omega(29)


def test_host_point_add_matches_oracle():
    rng = O.Rng(9)
    k = rng.fr_vector(6)
    pts = O.g1_fixed_base(k)
    for i in range(0, 6, 2):
        exp = O.msm_g1_naive(pts[i:i + 2], np.stack([O.fr_from_int(1)] * 2))
        assert np.array_equal(Z.g1_add_affine(pts[i], pts[i + 1]), exp)
    assert np.array_equal(Z.g1_add_affine(pts[0], np.zeros(8, np.uint64)), pts[0])
    assert np.array_equal(Z.g1_add_affine(pts[0], pts[0]), O.msm_g1_naive(pts[:1], O.fr_from_int(2)[None]))
    q = O.g2_fixed_base(k[:2])
    exp2 = O.msm_g2_naive(q, np.stack([O.fr_from_int(1)] * 2))
    assert np.array_equal(Z.g2_add_affine(q[0], q[1]), exp2)


def test_random_fr_is_canonical():
    v = Z.random_fr(10000, 3)
    assert all(Z.fr_to_int(x) < Z.R_MOD for x in v[:50])
    assert (v[:, 3] < np.uint64(Z.R_MOD >> 192)).all()


def test_compute_calls_fail_without_device():
    if Z.device_count() > 0:
        pytest.skip("a CUDA device is visible")
    pts = np.zeros((4, 8), np.uint64)
    sc = np.zeros((4, 4), np.uint64)
    with pytest.raises(Z.ZkError) as e:
        Z.msm_g1(pts, sc)
    assert e.value.status == Z.ZK_ERR_NODEV


def test_split_transform_and_pointwise_arguments_checked_first():
    """zk_ntt_cross_device and zk_compute_h_pointwise_device refuse bad shapes
    before they look for a device: ZK_ERR_RANGE / ZK_ERR_INVALID here, and
    ZK_ERR_NODEV (no CPU fallback) for valid shapes when no GPU is visible."""
    import ctypes
    buf = (ctypes.c_uint8 * 64)()
    other = (ctypes.c_uint8 * 64)()
    p, q = ctypes.cast(buf, ctypes.c_void_p), ctypes.cast(other, ctypes.c_void_p)
    cross = Z.lib.zk_ntt_cross_device
    for log_n, s_log, part, mode in ((8, 4, 0, 0), (8, 5, 0, 0), (8, 2, 4, 0), (8, 2, 0, 2), (8, -1, 0, 0), (3, 2, 0, 0)):
        assert cross(0, None, p, q, log_n, s_log, part, 0, mode, None, 0) == Z.ZK_ERR_RANGE, (log_n, s_log, part, mode)
    assert cross(0, None, p, p, 8, 1, 0, 0, 0, None, 0) == Z.ZK_ERR_INVALID  # in place
    assert cross(0, None, None, q, 8, 1, 0, 0, 0, None, 0) == Z.ZK_ERR_INVALID
    pw = Z.lib.zk_compute_h_pointwise_device
    assert pw(0, None, p, p, p, p, 4, 17) == Z.ZK_ERR_RANGE  # more values than the domain
    assert pw(0, None, None, p, p, p, 4, 4) == Z.ZK_ERR_INVALID
    if Z.device_count() == 0:
        assert cross(0, None, p, q, 8, 1, 0, 0, 0, None, 0) == Z.ZK_ERR_NODEV
        assert pw(0, None, p, p, p, p, 4, 16) == Z.ZK_ERR_NODEV
    assert Z.lib.zk_groth16_h_msm_blocks_device(None, None, p, 1, 0, p) == Z.ZK_ERR_INVALID


REF = O.reference_tree()


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "src")), reason="reference tree not present")
def test_reference_code_links_against_library(tmp_path):
    """A translation unit written against the reference's own headers
    (msm/msm.cuh, ntt/ntt.cuh) links against libzkml_b200.so alone, and the
    host-side entry point it can run here (compute_omega) returns the
    reference values."""
    src = tmp_path / "use_ref.cu"
    src.write_text(
        '#include "msm/msm.cuh"\n#include "ntt/ntt.cuh"\n#include <cstdio>\n'
        "using namespace bn254;\n"
        "int main(int argc, char** argv) {\n"
        "  if (argc > 5) { G1Affine p[1]; Fr s[1]; G1Jacobian r = msm_g1(p, s, 1);\n"
        "    G2Affine q[1]; G2Jacobian t = msm_g2(q, s, 1); ntt_gpu(s, s, 2, false); ntt_gpu_inplace(s, 2, true);\n"
        "    printf(\"%d %d\", (int)r.x.val[0], (int)t.x.c0.val[0]); }\n"
        "  for (int ln = 0; ln <= 28; ln++) { Fr w = compute_omega(ln), v = compute_omega_inv(ln);\n"
        "    printf(\"%016llx%016llx%016llx%016llx %016llx%016llx%016llx%016llx\\n\",\n"
        "      (unsigned long long)w.val[3], (unsigned long long)w.val[2], (unsigned long long)w.val[1], (unsigned long long)w.val[0],\n"
        "      (unsigned long long)v.val[3], (unsigned long long)v.val[2], (unsigned long long)v.val[1], (unsigned long long)v.val[0]); }\n"
        "  return 0; }\n")
    exe = tmp_path / "use_ref"
    libdir = os.path.dirname(Z.LIB_PATH)
    subprocess.run(["nvcc", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", f"-I{REF}/src", str(src), "-o", str(exe),
                    f"-L{libdir}", "-lzkml_b200", f"-Xlinker=-rpath,{libdir}"], check=True, capture_output=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    g = np.load(os.path.join(GOLDEN, "omega.npz"))
    for ln in range(29):
        w, v = out[ln].split()
        assert int(w, 16) == O.to_int(g["fwd"][ln])
        assert int(v, 16) == O.to_int(g["inv"][ln])


def test_msm_key_space_refused_before_device_work(monkeypatch):
    """Keys of the counting sort are counted and indexed in 32 bits.  A window
    width forced by ZK_MSM_WINDOW_BITS fixes the worst case n W before any
    device work, and a pass whose n W exceeds 2^31 - 1 is refused with
    ZK_ERR_RANGE (here, without a GPU, before the device lookup).  Larger MSMs
    with the automatic window run in passes of at most 2^27 points."""
    import ctypes
    buf = (ctypes.c_uint8 * 128)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    monkeypatch.setenv("ZK_MSM_WINDOW_BITS", "3")   # W = 85
    assert Z.lib.zk_msm_g1_device(0, None, p, p, (1 << 27), p) == Z.ZK_ERR_RANGE
    assert Z.lib.zk_msm_g1_host(0, None, p, p, (1 << 27) + 5, p) == Z.ZK_ERR_RANGE   # the first pass is refused
    assert "2^31" in Z.last_error()
    monkeypatch.setenv("ZK_MSM_G2_WINDOW_BITS", "4")  # W = 64
    assert Z.lib.zk_msm_g2_device(0, None, p, p, 1 << 25, p) == Z.ZK_ERR_RANGE   # 2^31 keys
    if Z.device_count() == 0:
        # within the key space the call goes on to the device lookup
        assert Z.lib.zk_msm_g2_device(0, None, p, p, (1 << 25) - 1, p) == Z.ZK_ERR_NODEV
        monkeypatch.delenv("ZK_MSM_WINDOW_BITS")
        assert Z.lib.zk_msm_g1_device(0, None, p, p, (1 << 27) + 5, p) == Z.ZK_ERR_NODEV


def test_split_prove_entry_points_check_arguments():
    """The C split prove's entry points refuse bad arguments before any device
    work; NCCL loads at run time (an id is made without a GPU); without a
    device the local communicator reports ZK_ERR_NODEV (no CPU fallback)."""
    import ctypes
    assert Z.lib.zk_groth16_prove_split(None, None, None, None, None, None, None, None) == Z.ZK_ERR_INVALID
    assert Z.lib.zk_groth16_prove_multi(None, None, None, 2, None, None, None, None, None, 1.0, None) == Z.ZK_ERR_INVALID
    hs = (ctypes.c_void_p * 2)()
    assert Z.lib.zk_comm_init_local(0, 0, ctypes.cast(hs, ctypes.c_void_p)) == Z.ZK_ERR_INVALID
    assert Z.lib.zk_comm_init_rank(0, None, 2, 0, None) == Z.ZK_ERR_INVALID
    assert Z.lib.zk_comm_abort(None) == Z.ZK_ERR_INVALID
    uid = Z.Comm.unique_id()
    assert len(uid) == 128 and uid != Z.Comm.unique_id()
    if Z.device_count() == 0:
        assert Z.lib.zk_comm_init_local(0, 2, ctypes.cast(hs, ctypes.c_void_p)) == Z.ZK_ERR_NODEV


def test_pk_load_refuses_bad_files_before_device_work(tmp_path):
    """zk_groth16_pk_load walks the ZKMLPK3 header and the five vector counts
    before it touches a device: a missing file, a wrong magic and a truncated
    key are refused with ZK_ERR_INVALID on a machine without a GPU; an intact
    key (the reference's own T4 pk.bin, read in place) passes the walk and then
    reports ZK_ERR_NODEV (no CPU fallback)."""
    import ctypes
    h = ctypes.c_void_p()
    assert Z.lib.zk_groth16_pk_load(0, str(tmp_path / "none.bin").encode(), ctypes.byref(h)) == Z.ZK_ERR_INVALID
    assert "cannot open" in Z.last_error()
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"ZKMLPK2\0" + bytes(64))
    assert Z.lib.zk_groth16_pk_load(0, str(bad).encode(), ctypes.byref(h)) == Z.ZK_ERR_INVALID
    assert "not a ZKMLPK3" in Z.last_error()
    ref_pk = os.path.join(O.reference_tree(), "results", "gpu_validation_2026", "artifacts", "p16", "pk.bin")
    if not os.path.exists(ref_pk):
        pytest.skip("reference artefacts not present")
    raw = open(ref_pk, "rb").read()
    cut = tmp_path / "cut.bin"
    cut.write_bytes(raw[:-100])
    assert Z.lib.zk_groth16_pk_load(0, str(cut).encode(), ctypes.byref(h)) == Z.ZK_ERR_INVALID
    assert "truncated" in Z.last_error()
    if Z.device_count() == 0:
        assert Z.lib.zk_groth16_pk_load(0, ref_pk.encode(), ctypes.byref(h)) == Z.ZK_ERR_NODEV
