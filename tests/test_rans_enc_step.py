"""The rANS encoders' step divides the state by the symbol frequency with a
64-bit reciprocal multiplication (csrc/common.cuh rans_enc_entry /
rans_enc_update); the step must equal (x / f) * M + (x mod f) + cum for every
precision, every frequency and any state the renormalisation leaves
(1 <= x < f * 2^(32-P)).  Host-only: compiled with nvcc as host code and run
on the CPU."""
from __future__ import annotations

import os
import shutil
import subprocess
import tempfile

import pytest

from tests.conftest import ROOT


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not available")
def test_rans_encode_step_matches_integer_arithmetic():
    with tempfile.TemporaryDirectory() as tmp:
        exe = os.path.join(tmp, "rans_enc_check")
        subprocess.run(["nvcc", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "bigsmall_b200", "csrc"),
                        "-I", os.path.join(ROOT, "include"), "-o", exe,
                        os.path.join(ROOT, "tests", "rans_enc_check.cu")], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, timeout=300)
        assert out.returncode == 0 and out.stdout.strip() == "ok", out.stdout + out.stderr
