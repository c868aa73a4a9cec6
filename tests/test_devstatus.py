"""Device status word watch (CPU, with a fake device word): the read is queued every n steps,
checked once ready, a nonzero code raises after clearing the word; the scheduler aborts the
requests in flight on it and keeps serving; a worker rank ends on it."""

import pytest

from fake_runner import FakeRunner
from qwen35_b200.parallel.driver import Op, serve_worker
from qwen35_b200.serving.block_pool import BlockAllocator
from qwen35_b200.serving.scheduler import Request, Scheduler
from qwen35_b200.serving.session_cache import SessionCache
from qwen35_b200.utils.devstatus import DeviceStatusError, StatusWatch


class FakeWord:
    def __init__(self):
        self.code = 0
        self.reads = 0
        self.cleared = 0
        self.ready = False

    def start(self):
        self.reads += 1
        value = self.code
        return (lambda: self.ready), (lambda: value)

    def clear(self):
        self.cleared += 1
        self.code = 0


def test_watch_reads_every_n_steps_and_raises_on_a_code():
    w = FakeWord()
    sw = StatusWatch(every=4, start=w.start, clear=w.clear)
    for _ in range(3):
        sw.step()
    assert w.reads == 0
    w.code = 5
    sw.step()  # 4th step queues a read (it sees code 5)
    assert w.reads == 1
    sw.step()  # not ready yet: nothing raised, no second read queued
    assert w.reads == 1
    w.ready = True
    with pytest.raises(DeviceStatusError, match="peer_wait"):
        sw.step()
    assert w.cleared == 1 and sw.pending is None
    StatusWatch(every=0, start=w.start, clear=w.clear).step()  # off


def test_scheduler_aborts_inflight_on_a_device_status_code():
    r = FakeRunner(max_batch=2, block_size=4)
    w = FakeWord()
    w.ready = True
    w.code = 1
    r.status_watch = StatusWatch(every=1, start=w.start, clear=w.clear)
    s = Scheduler(r, SessionCache(BlockAllocator(100, 4), 4, 4))
    ev = []
    s.submit(Request([1, 2, 3], 6, ev.append))
    s.run_until_idle()
    assert ev[-1][0] == "error" and "tma_wait" in ev[-1][1]
    ev2 = []
    s.submit(Request([1, 2, 3], 4, ev2.append))  # the word was cleared: serving goes on
    s.run_until_idle()
    assert ev2[-1][0] == "end"


class _Chan:
    def __init__(self, cmds):
        self.cmds = list(cmds)

    def recv(self):
        return self.cmds.pop(0)


def test_worker_ends_on_a_device_status_code():
    r = FakeRunner(max_batch=2, block_size=4)
    w = FakeWord()
    w.ready = True
    w.code = 5
    r.status_watch = StatusWatch(every=1, start=w.start, clear=w.clear)
    r.begin(0)
    r.attach_blocks(0, [1])
    cmds = [(Op.DECODE, ([0], [7], [0])), (Op.DECODE, ([0], [8], [1])), (Op.SHUTDOWN, ())]
    with pytest.raises(DeviceStatusError):
        serve_worker(r, _Chan(cmds))
