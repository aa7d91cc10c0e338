"""The persistent tensor-core GEMMs' tile assignment, checked on the host.

`csrc/tile_list.cuh` holds the function each CTA of `q8_tc_gemm_i8_kernel` and
`q8_tc_gemm_f32_kernel` calls to list its tiles, and the grid-size rule of
their launchers.  `tile_list_check.cpp` compiles that same header with the host
compiler and checks, over random expert-group layouts, list lengths and SM
counts, that every tile of a launch is listed by exactly one CTA with its
group's rows, and that no CTA's list is cut short.
"""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "..", "unlimited-ocr-kernel_b200", "csrc")


@pytest.mark.skipif(shutil.which("g++") is None, reason="no host C++ compiler")
def test_every_tile_listed_once(tmp_path):
    exe = str(tmp_path / "tile_list_check")
    subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-I", CSRC,
                    os.path.join(HERE, "tile_list_check.cpp"), "-o", exe], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ok"), r.stdout
