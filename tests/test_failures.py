"""Failure detection on the host (no GPU involved): a worker rank that dies flips /health to 503;
the command ring gives up instead of waiting forever when rank 0 goes quiet or a worker stops
reading; ranks booted with different lockstep flags refuse to serve together."""

import multiprocessing as mp
import os
import socket
import sys
import time

import psutil
import pytest
import requests

from qwen35_b200.parallel.driver import Op
from qwen35_b200.parallel.shm_channel import ShmChannel

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)


def test_worker_death_flips_health_to_503():
    from test_server import start, stop

    proc, url = start(tp=2)
    try:
        assert requests.get(url + "/health", timeout=5).status_code == 200
        kids = psutil.Process(proc.pid).children(recursive=True)
        workers = [k for k in kids if "--rank" in " ".join(k.cmdline())]
        assert workers, [k.cmdline() for k in kids]
        workers[0].kill()  # the rank leaves between steps: nothing of it is in flight
        code = None
        for _ in range(60):
            code = requests.get(url + "/health", timeout=5).status_code
            if code == 503:
                break
            time.sleep(0.5)
        assert code == 503
    finally:
        stop(proc)


def test_ring_reader_times_out_when_rank0_is_silent():
    name = f"qb_fail_{os.getpid()}_a"
    w = ShmChannel(name, 2, 0, size=4096, create=True)
    r = ShmChannel(name, 2, 1, timeout_s=0.2)
    t0 = time.perf_counter()
    with pytest.raises(TimeoutError, match="no command"):
        r.recv()
    assert time.perf_counter() - t0 < 5
    r.close()
    w.close()


def test_ring_writer_times_out_when_a_worker_stops_reading():
    name = f"qb_fail_{os.getpid()}_b"
    w = ShmChannel(name, 2, 0, size=4096, create=True, timeout_s=0.2)
    payload = "x" * 1000
    with pytest.raises(TimeoutError, match="stopped reading"):
        for _ in range(100):  # nobody reads: the ring fills, then the writer gives up
            w.send(Op.DECODE, (payload,))
    w.close()


def _handshake_rank(rank, port, impl, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      QB_MOE_IMPL=impl)
    import datetime

    import torch
    import torch.distributed as dist

    from qwen35_b200.models.config import tiny_config
    from qwen35_b200.models.qwen35 import Model
    from qwen35_b200.models.weights import random_weights
    from qwen35_b200.parallel.driver import PoolMismatchError, pool_handshake
    from qwen35_b200.parallel.plan import plan

    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    cfg = tiny_config()
    p = plan(cfg, rank, 2)
    m = Model(cfg, random_weights(cfg, p, "cpu", torch.float32, seed=0, with_mtp=False), p, dtype=torch.float32,
              max_batch=2, max_seq=128)
    try:
        pool_handshake(m)
        q.put((rank, "ok"))
    except PoolMismatchError:
        q.put((rank, "mismatch"))
    dist.destroy_process_group()


def test_ranks_with_different_lockstep_flags_refuse_to_serve():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_handshake_rank, args=(r, port, impl, q)) for r, impl in ((0, "mx"), (1, "f16"))]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert res == {0: "mismatch", 1: "mismatch"}


def _region_rank(rank, port, fail_stage, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2")
    import datetime

    import torch.distributed as dist

    from qwen35_b200.parallel.symm import SymmUnavailable, alloc_region

    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    freed, closed = [], []

    def alloc(n):
        if fail_stage == "alloc" and rank == 1:
            raise RuntimeError("out of device memory")
        return 1000 + rank, f"handle{rank}"

    def open_(h):
        if fail_stage == "open" and rank == 0:
            raise RuntimeError("peer access refused")
        return 2000 + int(h[-1])

    try:
        bases, own, opened = alloc_region(rank, 2, "cpu", 64, alloc=alloc, open_=open_, close=closed.append,
                                          free=freed.append)
        q.put((rank, "ok", bases))
    except SymmUnavailable:
        q.put((rank, "unavailable", (freed, closed)))
    dist.destroy_process_group()


@pytest.mark.parametrize("fail_stage", ["none", "alloc", "open"])
def test_symmetric_region_failure_on_one_rank_is_raised_on_every_rank(fail_stage):
    """A rank that cannot allocate or map the peer regions makes every rank raise at the same
    vote (so all fall back to NCCL together), with its own mappings undone; nobody waits."""
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_region_rank, args=(r, port, fail_stage, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {r: (st, info) for r, st, info in (q.get(timeout=120) for _ in ps)}
    for p in ps:
        p.join(timeout=60)
    if fail_stage == "none":
        assert res == {0: ("ok", [1000, 2001]), 1: ("ok", [2000, 1001])}
    elif fail_stage == "alloc":
        assert {r: st for r, (st, _) in res.items()} == {0: "unavailable", 1: "unavailable"}
    else:
        assert res[0] == ("unavailable", ([1000], [])) and res[1] == ("unavailable", ([1001], [2000]))
