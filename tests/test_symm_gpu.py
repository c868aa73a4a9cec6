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


def _world() -> int:
    """Ranks for the multi-GPU checks: every visible GPU, up to 8."""
    return min(torch.cuda.device_count(), 8)


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_multi_gpu_nvls_equals_nccl():
    """NVLS switch-reduced all-reduce + add + RMSNorm on every visible GPU (up to 8) against NCCL
    all-reduce + add + RMSNorm; skips when the fabric offers no multicast object."""
    world, port = _world(), _port()
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "nvls_rank.py"), str(r), str(world), str(port)])
             for r in range(world)]
    rcs = [p.wait(timeout=300) for p in procs]
    if all(rc == 3 for rc in rcs):
        pytest.skip("no NVLS multicast support on this fabric")
    assert rcs == [0] * world, rcs


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_fused_equals_nccl():
    """Every visible GPU (up to 8): the one-shot and sequence-parallel kernels against NCCL."""
    world, port = _world(), _port()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "symm_rank.py"), str(r), str(world), str(port)],
                              env=env) for r in range(world)]
    assert [p.wait(timeout=300) for p in procs] == [0] * world


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_multi_gpu_allgather_gemm_equals_allreduce_then_gemm():
    """Every visible GPU (up to 8): owner-only sequence-parallel all-reduce + the GEMM that pulls
    every rank's rows over NVLink against the full all-reduce + the plain GEMM."""
    world, port = _world(), _port()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "ag_rank.py"), str(r), str(world), str(port)],
                              env=env) for r in range(world)]
    assert [p.wait(timeout=300) for p in procs] == [0] * world


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_model_out_proj_fused_equals_unfused():
    """Tiny model on 2 or 4 ranks (its 4 DeltaNet key heads bound the split): a 1500-token
    prefill with the attention / DeltaNet out projections fused into the sequence-parallel
    all-reduce gives the same logits bit for bit."""
    world, port = (4 if _world() >= 4 else 2), _port()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "sp_model_rank.py"), str(r), str(world), str(port)],
                              env=env) for r in range(world)]
    assert [p.wait(timeout=300) for p in procs] == [0] * world


def test_expert_parallel_one_rank_equals_local_moe():
    """Expert-parallel dispatch / experts / combine with one rank (every token's row goes to
    itself through the receive area) equals the local routed-expert op, over consecutive calls
    (parity halves reused) and token counts from 0 to the area's capacity."""
    from qwen35_b200.ops import core as ops
    from qwen35_b200.ops._ext import ext
    from qwen35_b200.parallel.ep import EPComm
    from qwen35_b200.utils import mxfp4

    dev = torch.device("cuda", 0)
    E, k, H, I = 16, 4, 512, 256
    g = torch.Generator(device=dev).manual_seed(3)
    w13, s13 = mxfp4.quantize(torch.randn(E, 2 * I, H, device=dev, generator=g) * 0.02)
    w2, s2 = mxfp4.quantize(torch.randn(E, H, I, device=dev, generator=g) * 0.02)
    full = {"w13": w13, "s13": s13, "w2": w2, "s2": s2}
    ep = EPComm(0, 1, dev, cap=128, hidden=H, top_k=k, experts=E)
    ext().clear_status(torch.empty(1, device=dev))
    for T in (5, 128, 0, 77, 1):
        h = torch.randn(T, H, device=dev, generator=g).bfloat16()
        tw, ti = ops.router_topk(torch.randn(T, E, device=dev, generator=g).bfloat16(), k)
        y = ep.moe(h, tw, ti, {kk: v.clone() for kk, v in full.items()})
        ref = ops.moe_routed(h, tw, ti, {kk: v.clone() for kk, v in full.items()}, 0, E)
        torch.cuda.synchronize()
        assert y.shape == (T, H)
        if T:
            assert (y.float() - ref.float()).abs().max().item() <= 1e-2 * ref.float().abs().max().item() + 1e-3
    assert ext().status(torch.empty(1, device=dev)).tolist()[0] == 0
    ep.close()


def test_expert_parallel_silent_peer_times_out_cleanly():
    """A peer that never dispatches: the receive and combine waits give up within the bound,
    the status word says ERR_PEER_WAIT, the output is finite and the GPU stays usable."""
    from qwen35_b200.ops import core as ops
    from qwen35_b200.ops._ext import ext
    from qwen35_b200.parallel.ep import EPComm
    from qwen35_b200.utils import mxfp4

    dev = torch.device("cuda", 0)
    E, k, H, I = 16, 2, 256, 128
    nbytes = ext().ep_region_bytes(2, 32, H, k)
    own, _ = ext().symm_alloc(nbytes)
    fake_peer, _ = ext().symm_alloc(nbytes)  # a local region standing in for a silent peer
    ep = EPComm(0, 2, dev, cap=32, hidden=H, top_k=k, experts=E, bases=[own, fake_peer], timeout_s=0.05)
    w13, s13 = mxfp4.quantize(torch.randn(E // 2, 2 * I, H, device=dev) * 0.02)
    w2, s2 = mxfp4.quantize(torch.randn(E // 2, H, I, device=dev) * 0.02)
    ext().clear_status(torch.empty(1, device=dev))
    h = torch.randn(8, H, device=dev).bfloat16()
    tw, ti = ops.router_topk(torch.randn(8, E, device=dev).bfloat16(), k)
    y = ep.moe(h, tw, ti, {"w13": w13, "s13": s13, "w2": w2, "s2": s2})
    torch.cuda.synchronize()
    assert ext().status(torch.empty(1, device=dev)).tolist()[0] == 5  # ERR_PEER_WAIT
    ext().clear_status(torch.empty(1, device=dev))
    assert torch.isfinite(y.float()).all()
    z = ops.rmsnorm(h, torch.ones(H, device=dev), 1e-6)  # the context is still usable
    torch.cuda.synchronize()
    assert torch.isfinite(z.float()).all()
    ext().symm_free(own)
    ext().symm_free(fake_peer)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_expert_parallel_equals_local():
    world, port = _world(), _port()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "ep_rank.py"), str(r), str(world), str(port)],
                              env=env) for r in range(world)]
    assert [p.wait(timeout=300) for p in procs] == [0] * world
