"""In-tree build of the sm_100a extension (``_build/qwen35_b200_C*.so``).

Compiled with ``-gencode arch=compute_100a,code=sm_100a`` (passing ``-gencode`` explicitly
keeps PyTorch from adding its own architecture list). Run on a machine without a GPU it
cross-compiles; the ``.so`` is loaded by path at runtime (``ops._ext``), never rebuilt there.
"""

from __future__ import annotations

import glob
import os

from ._ext import BUILD_DIR, MODULE_NAME

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


def build(verbose: bool = False):
    import torch.utils.cpp_extension as ce

    os.makedirs(BUILD_DIR, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    os.environ.setdefault("MAX_JOBS", str(min(8, os.cpu_count() or 4)))
    return ce.load(
        name=MODULE_NAME,
        sources=sources(),
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=CUDA_FLAGS,
        extra_include_paths=[CSRC],
        build_directory=BUILD_DIR,
        verbose=verbose,
        with_cuda=True,
    )
