"""The sensitivity kernel replaces w*w / h by a reciprocal and two fused
corrections; this checks, exhaustively on the CPU, that the result is the
correctly rounded quotient for every possible dividend (the square of any
fp16 value) and every fp32 divisor significand (tests/division_check.c)."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def test_fma_corrected_division_is_correctly_rounded(tmp_path):
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("no C compiler")
    flags = ["-O3", "-ffp-contract=off", "-pthread"]
    if "fma" in open("/proc/cpuinfo").read().split():
        flags.append("-mfma")  # hardware fmaf; libm's is exact either way, only slower
    exe = str(tmp_path / "division_check")
    subprocess.run([cc, *flags, os.path.join(HERE, "division_check.c"), "-o", exe, "-lm"],
                   check=True)
    r = subprocess.run([exe, str(os.cpu_count() or 8)], capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "mismatches 0" in r.stdout
