"""The device softmax's expf formula (exact_expf.h) against the host C library.

The reference's routing softmax calls the host expf (engine/src/model.c:1031,
:312); bit-exact routing weights need the same values on the device. This
compiles exact_expf.h as host C and compares all 2^31 non-positive floats
(routing only evaluates expf(l - max) with l <= max). The GPU test
test_gpu_route.py::test_device_expf_matches_host checks the device build.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_exact_expf_exhaustive(tmp_path):
    exe = tmp_path / "expf_check"
    src = os.path.join(ROOT, "tests", "native", "expf_check.c")
    inc = os.path.join(ROOT, "ornith-flight_b200", "csrc")
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-fopenmp", "-I", inc, src, "-o", str(exe),
                    "-lm"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert r.stdout.strip() == "0", f"mismatches: {r.stdout}"
    assert r.returncode == 0
