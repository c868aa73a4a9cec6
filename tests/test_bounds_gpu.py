"""The debug build (-DQB_BOUNDS): index checks and scratch canaries record into the device status
word instead of faulting (child process: the debug extension is loaded instead of the release one)."""

import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
BOUNDS_DIR = os.path.join(os.path.dirname(HERE), "qwen3.5-397b-mi300a-bespoke-vibesys-20260920_b200", "_build_bounds")


@pytest.mark.gpu
def test_bounds_build_records_out_of_range_indices():
    import glob

    if not glob.glob(os.path.join(BOUNDS_DIR, "qwen35_b200_C*.so")):
        pytest.skip("debug build not present (python -m qwen35_b200.ops.build --bounds)")
    env = dict(os.environ, QB_BOUNDS="1")
    r = subprocess.run([sys.executable, os.path.join(HERE, "bounds_check.py")], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "bounds ok" in r.stdout
