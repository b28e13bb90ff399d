"""The division-free requantization's arithmetic, restated in C and checked on
the CPU against an IEEE division and roundf (tests/native/requant_check.c):
one scale's whole input range, the neighbourhood of every rounding tie for
300 scales, random and special values, and the rounding over a stride of all
bit patterns. The GPU side of the same claim is test_gpu_requant.py."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_requant_quotient_and_rounding(tmp_path):
    exe = tmp_path / "requant_check"
    src = os.path.join(HERE, "native", "requant_check.c")
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-o", str(exe), src, "-lm"], check=True)
    r = subprocess.run([str(exe), "300"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "mismatches 0, int8 mismatches 0, rounding mismatches 0" in r.stdout, r.stdout
