"""Fused one-shot all-reduce + residual + RMSNorm over peer memory.

* single GPU: a rank whose peer never publishes must time out within the bound, report
  ``ERR_PEER_WAIT`` in the status word and leave the GPU usable (no trap, no hang);
* two GPUs (when visible): the fused kernel equals NCCL all-reduce + add + RMSNorm, over many
  consecutive calls (epoch and slot reuse) and under CUDA-graph replay.
"""

import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_peer_that_never_signals_times_out_cleanly():
    from qwen35_b200.ops import core as ops
    from qwen35_b200.ops._ext import ext
    from qwen35_b200.parallel.symm import SymmComm

    dev = torch.device("cuda", 0)
    nbytes = SymmComm.region_bytes(64, 256)
    own, _ = ext().symm_alloc(nbytes)
    fake_peer, _ = ext().symm_alloc(nbytes)  # a local region standing in for a silent peer
    s = SymmComm(0, 2, dev, 64, 256, bases=[own, fake_peer], timeout_s=0.05)
    ext().clear_status(torch.empty(1, device=dev))
    x = torch.randn(8, 256, device=dev).bfloat16()
    res = torch.randn(8, 256, device=dev).bfloat16()
    w = torch.ones(256, device=dev)
    s.allreduce_add_rmsnorm(x, res, w, 1e-6)
    torch.cuda.synchronize()
    st = ext().status(torch.empty(1, device=dev)).tolist()
    assert st[0] == 5, st  # ERR_PEER_WAIT
    ext().clear_status(torch.empty(1, device=dev))
    y = ops.rmsnorm(x, w, 1e-6)  # the context is still usable
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
    ext().symm_free(own)
    ext().symm_free(fake_peer)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_fused_equals_nccl():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "symm_rank.py"), str(r), "2", str(port)], env=env)
             for r in range(2)]
    assert [p.wait(timeout=300) for p in procs] == [0, 0]
