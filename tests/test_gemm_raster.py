"""The persistent GEMM's tile order (gemm_raster.cuh, the function the kernel
calls, compiled for the host): every output tile exactly once for every grid up to
96 x 96 tiles and every panel width, panels swept in order."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_raster_covers_every_tile_once(tmp_path):
    exe = str(tmp_path / "raster_check")
    subprocess.run(["g++", "-O2", "-std=c++17", "-o", exe, os.path.join(ROOT, "tests", "raster_check.cpp"),
                    "-I", os.path.join(ROOT, "welvet.metal_b200", "csrc")], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert " 0 mismatches" in r.stdout
