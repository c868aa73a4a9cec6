"""Shared pytest setup: the ``gpu`` marker, the repo on ``sys.path``, and session fixtures."""

from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and the built extension")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def tiny_dir(tmp_path_factory):
    """The tiny parity checkpoint (hidden 256, 8 layers, 32 experts, MXFP4 experts, seed 0)."""
    from qwen35_b200.models.config import tiny_config
    from qwen35_b200.models.weights import write_tiny_checkpoint

    d = tmp_path_factory.mktemp("tiny")
    write_tiny_checkpoint(str(d), tiny_config(), seed=0)
    return str(d)
