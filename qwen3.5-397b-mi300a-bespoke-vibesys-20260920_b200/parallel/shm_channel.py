"""Shared-memory command ring between rank 0 and the other ranks of one node.

The gloo broadcast used by ``driver.Channel`` costs a network round trip per command, and rank
0 cannot start a step's collectives before every worker has received that step's command, so
its latency lands on every step. This ring lives in ``/dev/shm``: rank 0 appends
``[u32 length][payload]`` records and advances a 64-bit write counter; each worker polls the
counter, copies its record and advances its own read counter. Rank 0 blocks only when it would
overwrite a record some worker has not read yet. Records never wrap: if one does not fit in the
remaining space, a zero-length marker sends readers back to offset 0.

Layout: [write_seq u64][read_seq u64 x world][pad to 4 KiB][ring bytes]. ``write_seq`` and each
``read_seq`` count bytes consumed since the start (monotonic), so positions are ``seq % size``.
"""

from __future__ import annotations

import atexit

import pickle
import struct
import time
from multiprocessing import shared_memory

import numpy as np

from .driver import Op

HEADER = 4096


class ShmChannel:
    def __init__(self, name: str, world: int, rank: int, size: int = 64 << 20, create: bool = False,
                 poll_s: float = 0.0, timeout_s: float = 3600.0):
        self.world, self.rank, self.size = world, rank, size
        if create:
            self.shm = shared_memory.SharedMemory(name=name, create=True, size=HEADER + size)
            self.shm.buf[:HEADER] = bytes(HEADER)
        else:
            # only the creator owns the segment: a reader attaches without registering it with
            # the resource tracker, which would otherwise unlink it at the reader's exit too (and
            # warn about a "leaked" segment the creator already removed)
            from multiprocessing import resource_tracker

            register = resource_tracker.register
            resource_tracker.register = lambda *a, **k: None
            try:
                self.shm = shared_memory.SharedMemory(name=name)
            finally:
                resource_tracker.register = register
        self.ctr = np.ndarray((1 + world,), dtype=np.uint64, buffer=self.shm.buf[:8 * (1 + world)])
        self.ring = self.shm.buf[HEADER:HEADER + size]
        self._closed = False
        atexit.register(self.close)
        self.poll_s = poll_s
        self.timeout_s = timeout_s
        self.owner = create

    # ------------------------------------------------------------------ rank 0
    def _wait_space(self, need: int) -> None:
        t0 = time.perf_counter()
        while True:
            w = int(self.ctr[0])
            slow = min(int(self.ctr[1 + r]) for r in range(1, self.world)) if self.world > 1 else w
            if w + need - slow <= self.size:
                return
            if time.perf_counter() - t0 > self.timeout_s:
                raise TimeoutError("command ring full: a worker stopped reading")
            time.sleep(0)

    def send(self, op: Op, args: tuple) -> None:
        raw = pickle.dumps((int(op), args), protocol=pickle.HIGHEST_PROTOCOL)
        rec = 4 + len(raw)
        if rec + 4 > self.size:
            raise ValueError("command larger than the ring")
        w = int(self.ctr[0])
        pos = w % self.size
        if pos + rec > self.size:  # does not fit before the end: wrap marker, restart at 0
            self._wait_space(self.size - pos)
            if self.size - pos >= 4:
                self.ring[pos:pos + 4] = struct.pack("<I", 0)
            w += self.size - pos
            self.ctr[0] = np.uint64(w)
            pos = 0
        self._wait_space(rec)
        self.ring[pos:pos + 4] = struct.pack("<I", len(raw))
        self.ring[pos + 4:pos + rec] = raw
        self.ctr[0] = np.uint64(w + rec)  # publish after the payload is in place

    # ------------------------------------------------------------------ workers
    def recv(self):
        me = 1 + self.rank
        t0 = time.perf_counter()
        while True:
            r = int(self.ctr[me])
            if int(self.ctr[0]) > r:
                pos = r % self.size
                if self.size - pos < 4:
                    self.ctr[me] = np.uint64(r + self.size - pos)
                    continue
                (n,) = struct.unpack("<I", bytes(self.ring[pos:pos + 4]))
                if n == 0:  # wrap marker
                    self.ctr[me] = np.uint64(r + self.size - pos)
                    continue
                raw = bytes(self.ring[pos + 4:pos + 4 + n])
                self.ctr[me] = np.uint64(r + 4 + n)
                op, args = pickle.loads(raw)
                return Op(op), args
            if time.perf_counter() - t0 > self.timeout_s:
                raise TimeoutError("no command from rank 0")
            if self.poll_s:
                time.sleep(self.poll_s)

    def close(self) -> None:
        """Release the views, unmap (and unlink, for the creator). Idempotent; also registered
        with ``atexit``, since unmapping at interpreter teardown with live views fails."""
        if getattr(self, "_closed", True):
            return
        self._closed = True
        del self.ctr
        self.ring.release()
        self.shm.close()
        if self.owner:
            try:
                self.shm.unlink()
            except FileNotFoundError:
                pass


def make_channel(world: int, rank: int, group) -> ShmChannel | None:
    """Rank 0 creates the ring and broadcasts its name over ``group``; everyone attaches."""
    if world <= 1:
        return None
    import os

    import torch.distributed as dist

    name = [f"qb_cmd_{os.getpid()}_{int(time.time() * 1e3) % 100000}" if rank == 0 else None]
    ch = ShmChannel(name[0], world, rank, create=True) if rank == 0 else None
    dist.broadcast_object_list(name, src=0, group=group)
    if rank != 0:
        ch = ShmChannel(name[0], world, rank)
    dist.barrier(group=group)
    return ch
