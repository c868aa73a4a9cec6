"""In-tree build of the sm_100a extension (``_build/qwen35_b200_C*.so``).

Compiled with ``-gencode arch=compute_100a,code=sm_100a`` (passing ``-gencode`` explicitly
keeps PyTorch from adding its own architecture list). Run on a machine without a GPU it
cross-compiles; the ``.so`` is loaded by path at runtime (``ops._ext``), never rebuilt there.
"""

from __future__ import annotations

import glob
import os

from ._ext import BOUNDS_BUILD_DIR, BUILD_DIR, MODULE_NAME

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(PKG, "csrc")

CUDA_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-O3",
]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))


def build(verbose: bool = False, bounds: bool = False):
    """The release extension, or with ``bounds=True`` the debug build (``-DQB_BOUNDS``: index checks
    and scratch canaries that record into the device status word, ``csrc/bounds.cuh``) in
    ``_build_bounds/``, which ``ops._ext`` loads instead when ``QB_BOUNDS=1``."""
    import torch.utils.cpp_extension as ce

    build_dir = BOUNDS_BUILD_DIR if bounds else BUILD_DIR
    os.makedirs(build_dir, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    os.environ.setdefault("MAX_JOBS", str(min(8, os.cpu_count() or 4)))
    return ce.load(
        name=MODULE_NAME + ("_bounds" if bounds else ""),
        sources=sources(),
        extra_cflags=["-O3", "-std=c++17"] + (["-DQB_BOUNDS"] if bounds else []),
        extra_cuda_cflags=CUDA_FLAGS + (["-DQB_BOUNDS"] if bounds else []),
        extra_include_paths=[CSRC],
        build_directory=build_dir,
        verbose=verbose,
        with_cuda=True,
    )


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description="build the sm_100a extension in-tree")
    ap.add_argument("--bounds", action="store_true", help="the debug build with bounds checks and canaries")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    build(verbose=a.verbose, bounds=a.bounds)
