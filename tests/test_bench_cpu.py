"""bench.py's output contract on CPU: the reference arm (the reference's own
CPU kernel, oracle/_ref) prints exactly one JSON line on stdout carrying the
keys a driver reads, whatever else the process writes; and the algorithmic
byte counts the GPU arm reports follow from the block sizes."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_json_line():
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, res.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    if "unavailable" in d:
        pytest.skip(d["unavailable"])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1


def test_step_and_projection_bytes():
    sys.path.insert(0, ROOT)
    import bench
    # the sweep: 8 matrices of 4096 x 11008 (either orientation), packed rows + x + y
    per_type = {"Q8_0": 34 / 32, "Q4_K": 144 / 256, "Q5_K": 176 / 256, "Q6_K": 210 / 256}
    w = sum(2 * 4096 * 11008 * bpw for bpw in per_type.values())
    xy = 4 * 2 * (4096 + 11008) * 4
    assert bench.step_bytes() == int(w) + xy
    # the 70B projection set at one and at eight ranks: x is read once per rank
    q4k = 144 / 256
    mats = bench.PROJ70B
    weights = sum(int(n * k * q4k) for _, n, k in mats)
    assert bench.proj70b_bytes(1) == weights + sum(4 * (n + k) for _, n, k in mats)
    assert bench.proj70b_bytes(8) - bench.proj70b_bytes(1) == 7 * sum(4 * k for _, _, k in mats)
