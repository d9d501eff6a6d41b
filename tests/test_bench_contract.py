"""bench.py's reference arm on the CPU: one JSON line with the driver's keys.

Runs `bench.py --impl reference` on a small sample (the reference's Pippenger
schedule on its own host arithmetic from oracle/_ref, or the oracle port where
that is not built); the GPU legs of the arm (the reference's ntt_gpu and its
prover linked against this library) need a device and are absent here."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0",
                          "--ref-sample", "4096"], capture_output=True, text=True, timeout=600, cwd=ROOT,
                         env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling", "dtype",
              "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["metric"] == "G1 MSM points/s @2^24" and d["unit"] == "points/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["host"]["nproc"] >= 1
    if cb["kind"] == "reference":
        nv = d["reference_naive_msm"]
        assert nv["points"] == 1 << 16 and nv["points_per_s"] > 0


@pytest.mark.parametrize("rank", ["1"])
def test_reference_arm_other_ranks_exit_quietly(rank):
    """Under torchrun only rank 0 runs and prints the reference arm."""
    env = {**os.environ, "CUDA_VISIBLE_DEVICES": "", "RANK": rank, "WORLD_SIZE": "2", "LOCAL_RANK": rank}
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "1",
                          "--warmup", "0", "--ref-sample", "4096"], capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    assert not [l for l in out.stdout.splitlines() if l.startswith("{")]
