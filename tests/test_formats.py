"""The ZKMLPK3 / vk.bin reader used by the GPU tests, pinned against the
reference's own committed T4 artefacts (read in place when the reference tree
is present; nothing is copied)."""
import os

import pytest

import pyoracle
import zkmlpk3

REF = pyoracle.reference_tree()
ART = os.path.join(REF, "results", "gpu_validation_2026", "artifacts")


@pytest.mark.skipif(not os.path.isdir(ART), reason="reference artefacts not present")
@pytest.mark.parametrize("case", ["p16", "p160"])
def test_parse_reference_proving_key(case):
    path = os.path.join(ART, case, "pk.bin")
    if not os.path.exists(path):
        pytest.skip("no pk.bin for " + case)
    buf = open(path, "rb").read()
    key = zkmlpk3.parse_pk(buf)
    assert len(buf) == zkmlpk3.pk_size(len(key["H"]), key["m"], len(key["L"]), len(key["tau_g2"]), len(key["tau_g1"]))
    assert len(key["A"]) == len(key["B1"]) == len(key["B2"]) == key["m"]
    assert len(key["H"]) == key["n"]
    assert len(key["L"]) == key["m"] - key["num_public"] - 1
    # points are on the curve y^2 = x^3 + 3
    P = zkmlpk3.P
    for pt in key["A"][:50] + [key["alpha1"], key["beta1"], key["delta1"]]:
        if pt is not None:
            x, y = pt
            assert (y * y - x * x * x - 3) % P == 0


def test_p160_size_formula():
    # p160 (n = 1024, m = 716, pub = 75, L = 640) is 294,496 bytes
    assert zkmlpk3.pk_size(1024, 716, 640) == 294496


@pytest.mark.skipif(not os.path.isdir(ART), reason="reference artefacts not present")
def test_parse_reference_vk():
    path = os.path.join(ART, "p160", "vk.bin")
    if not os.path.exists(path):
        pytest.skip("no vk.bin")
    vk = zkmlpk3.parse_vk(open(path, "rb").read())
    assert len(vk["ic"]) == vk["num_public"] + 1
