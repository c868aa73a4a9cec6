"""Native host tests: `tests/native/host_numerics.cpp` compiled with the host C++ compiler checks
the kernels' bit-exact numeric helpers (`csrc/numerics.cuh`) exhaustively or on large random
samples: e2m1 code placement of the f16-decode MoE path, the exact hi/lo e4m3 split of the
block-scaled path (exact for every element within 2^13 of its block maximum) and the scale-chunk
layout. Runs without a GPU."""

import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "..", "qwen3.5-397b-mi300a-bespoke-vibesys-20260920_b200", "csrc")


def test_host_numerics(tmp_path):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no host C++ compiler")
    exe = str(tmp_path / "host_numerics")
    subprocess.run([cxx, "-O2", "-std=c++17", "-I", CSRC, os.path.join(HERE, "native", "host_numerics.cpp"), "-o",
                    exe], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().startswith("ok"), r.stdout
