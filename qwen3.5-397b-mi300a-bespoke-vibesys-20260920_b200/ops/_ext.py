"""Loader of the compiled sm_100a extension.

The extension is built in-tree by ``ops.build.build()`` (``__graft_entry__.build`` calls it)
into ``_build/qwen35_b200_C*.so`` next to the package sources, and loaded from there by path:
no JIT build happens at import, and nothing is installed into site-packages. On a CUDA tensor
every op requires the extension; if it is missing, ``ext()`` raises instead of falling back.
"""

from __future__ import annotations

import glob
import importlib.util
import os
import threading

import torch

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILD_DIR = os.path.join(_PKG, "_build")
BOUNDS_BUILD_DIR = os.path.join(_PKG, "_build_bounds")  # debug build (-DQB_BOUNDS), loaded when QB_BOUNDS=1
MODULE_NAME = "qwen35_b200_C"

_lock = threading.Lock()
_mod = None


def so_path() -> str | None:
    from ..utils import flags

    d = BOUNDS_BUILD_DIR if flags.get("QB_BOUNDS") else BUILD_DIR
    hits = sorted(glob.glob(os.path.join(d, MODULE_NAME + "*.so")))
    return hits[0] if hits else None


def available() -> bool:
    try:
        ext()
        return True
    except Exception:
        return False


def ext():
    """The loaded extension module (raises ``RuntimeError`` if it was not built)."""
    global _mod
    if _mod is not None:
        return _mod
    with _lock:
        if _mod is not None:
            return _mod
        path = so_path()
        if path is None:
            raise RuntimeError(
                f"qwen35_b200 CUDA extension not built (expected {BUILD_DIR}/{MODULE_NAME}*.so); "
                "run `python -c 'import __graft_entry__ as g; g.build()'`"
            )
        torch.cuda.init() if torch.cuda.is_available() else None
        # the module's own name: the file stem (the debug build is qwen35_b200_C_bounds)
        spec = importlib.util.spec_from_file_location(os.path.basename(path).split(".")[0], path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _mod = mod
        return _mod
