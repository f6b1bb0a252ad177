"""The FormatNone round trips of the device kernels (formatnone.cuh, the same
source compiled for the host) against the C restatement of the reference's
WeightStore round trip, on a strided sample of every FP32 bit pattern and of
five value ranges. `formatnone_check 1` enumerates every input (hours)."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE = os.path.join(ROOT, "oracle")


def test_formatnone_device_formulas_match_oracle(tmp_path):
    lib = os.path.join(ORACLE, "liboracle.so")
    if not os.path.exists(lib):
        pytest.skip("oracle/liboracle.so not built")
    exe = str(tmp_path / "formatnone_check")
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-o", exe,
                    os.path.join(ROOT, "tests", "formatnone_check.cpp"),
                    "-I", os.path.join(ROOT, "welvet.metal_b200", "csrc"),
                    "-L", ORACLE, "-loracle", f"-Wl,-rpath,{ORACLE}"], check=True)
    r = subprocess.run([exe, "1021"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert r.stdout.count(" 0 mismatches") == 34
