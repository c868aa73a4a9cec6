"""The shared-memory command ring: ordering, wrap-around, large records, back-pressure."""

import multiprocessing as mp
import os

from qwen35_b200.parallel.driver import Op
from qwen35_b200.parallel.shm_channel import ShmChannel


def _reader(name, world, rank, n, q):
    ch = ShmChannel(name, world, rank, size=4096)
    got = [ch.recv() for _ in range(n)]
    q.put((rank, [(int(op), a) for op, a in got]))
    ch.close()


def test_ring_delivers_in_order_with_wrap_and_backpressure():
    name = f"qb_test_{os.getpid()}"
    world, n = 3, 300
    w = ShmChannel(name, world, 0, size=4096, create=True)
    q = mp.get_context("spawn").Queue()
    ps = [mp.get_context("spawn").Process(target=_reader, args=(name, world, r, n, q)) for r in (1, 2)]
    for p in ps:
        p.start()
    sent = []
    for i in range(n):
        args = (i, list(range(i % 97)), "x" * (i % 50))  # varying sizes force wrap-around
        w.send(Op.DECODE, args)
        sent.append((int(Op.DECODE), args))
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    w.close()
    assert res[1] == sent and res[2] == sent
