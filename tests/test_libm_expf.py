"""The device's exp for REFERENCE numerics (wginfer_b200/csrc/libm_expf.cuh)
restates the C library's expf. Compiled here as host code, it must give the
host expf's exact result on every one of the 2^32 single-precision inputs.
(The device compiles the same header: fused multiply-adds, products and the
double-to-float rounding are IEEE-exact operations on both, and
test_ops_gpu.py::test_swiglu_f32_reference_exp_sweep checks the device.)"""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "wginfer_b200", "csrc")


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_expf_restatement_matches_libc_on_all_inputs(tmp_path):
    exe = str(tmp_path / "expf_exhaustive")
    subprocess.check_call(["g++", "-O2", "-fopenmp", "-ffp-contract=off", "-I", CSRC, "-o", exe,
                           os.path.join(HERE, "expf_exhaustive.cpp"), "-lm"])
    r = subprocess.run([exe, "1"], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "checked 4294967296 differ 0" in r.stdout
