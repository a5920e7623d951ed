"""CPU check that the GPU cast's fp32 division shortcut (quantize.cuh,
CastMarkstein) equals IEEE division for every bf16 significand against every fp32
scale significand, and across exponents at the edges of the scale window where
the kernel uses it; and that the form without the clamp (current scaling of a
tensor without NaN) gives the reference bytes for every |x| <= amax.  The C
program is compiled with gcc and run here."""

from __future__ import annotations

import os
import shutil
import subprocess

import pytest

SRC = os.path.join(os.path.dirname(__file__), "quantize_division_check.c")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_markstein_division_is_exact(tmp_path):
    exe = str(tmp_path / "qd")
    base = ["gcc", "-O2", "-ffp-contract=off", SRC, "-o", exe, "-lm"]
    if subprocess.run(base[:3] + ["-fopenmp"] + base[3:], capture_output=True).returncode != 0:
        subprocess.run(base, check=True, capture_output=True)
    out = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "mismatches 0; exponent sweep" in out.stdout and out.stdout.strip().endswith("mismatches 0")
    assert "no-clamp bytes" in out.stdout
