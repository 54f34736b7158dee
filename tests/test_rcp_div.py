"""The rANS encoders' divide-by-frequency uses Granlund-Montgomery division
by an invariant integer (csrc/common.cuh rcp_div); its result must equal
integer division for every divisor the encoders can see (frequencies
1..2^12, checked up to 2^16) and any 32-bit state.  Host-only: compiled with
nvcc as host code and run on the CPU."""
from __future__ import annotations

import os
import shutil
import subprocess
import tempfile

import pytest

from tests.conftest import ROOT


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not available")
def test_rcp_div_matches_integer_division():
    with tempfile.TemporaryDirectory() as tmp:
        exe = os.path.join(tmp, "rcp_div_check")
        subprocess.run(["nvcc", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "bigsmall_b200", "csrc"),
                        "-I", os.path.join(ROOT, "include"), "-o", exe,
                        os.path.join(ROOT, "tests", "rcp_div_check.cu")], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, timeout=300)
        assert out.returncode == 0 and out.stdout.strip() == "ok", out.stdout + out.stderr
