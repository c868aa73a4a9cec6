"""Benchmark harness self-test (host only): the closed-loop multi-turn chat driver over the real
scheduler and session cache with the deterministic fake runner."""

from fake_runner import FakeRunner
from qwen35_b200.serving.block_pool import BlockAllocator
from qwen35_b200.serving.scheduler import Scheduler
from qwen35_b200.serving.session_cache import SessionCache
from qwen35_b200.serving.workload import ChatSpec, ClosedLoop, percentile


def _run(spec):
    r = FakeRunner(max_batch=4, num_snapshots=32, block_size=4)
    s = Scheduler(r, SessionCache(BlockAllocator(4000, 4), 4, 32))
    loop = ClosedLoop(s, spec)
    loop.start()
    peak = len(loop.active)
    while loop.active:
        s.step()
        loop.pump()
        peak = max(peak, len(loop.active))
    return loop, peak


def test_closed_loop_shape_and_determinism():
    spec = ChatSpec(sessions=6, concurrency=3, turns=3, first_len=(20, 40), user_len=(5, 10), gen_len=(4, 8),
                    vocab=900, seed=0)
    loop, peak = _run(spec)
    assert peak == 3 and loop.finished_sessions == 6
    recs = sorted(loop.records, key=lambda r: (r.session, r.turn))
    assert len(recs) == 18 and all(r.error is None for r in recs)
    for r in recs:
        assert r.generated == r.max_new and 4 <= r.max_new <= 8  # EOS ignored: every token generated
        if r.turn == 0:
            assert 20 <= r.prompt_len <= 40
    for a, b in zip(recs, recs[1:]):
        if a.session == b.session:  # each turn extends the full prior history
            assert 5 <= b.prompt_len - (a.prompt_len + a.generated) <= 10
            assert b.reused >= a.prompt_len  # later turns hit the session cache
    again, _ = _run(spec)
    assert [(r.session, r.turn, r.prompt_len, r.max_new) for r in sorted(again.records, key=lambda r: (r.session, r.turn))] \
        == [(r.session, r.turn, r.prompt_len, r.max_new) for r in recs]


def test_percentile():
    assert percentile([], 50) != percentile([], 50)  # nan
    assert percentile([1.0, 2.0, 3.0, 4.0], 50) == 2.5
    assert percentile([5.0], 95) == 5.0
    assert abs(percentile(list(map(float, range(101))), 95) - 95.0) < 1e-9


def test_defaults_are_the_named_workload():
    """The chat workload's defaults, and bench.py's, are the configuration the headline is quoted
    on: 256 sessions at concurrency 32, 6 turns, a 2000-8000-id first prompt, 200-1000 new ids per
    later turn, 200-500 generated tokens per turn, seed 0."""
    import os
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench

    s = ChatSpec()
    assert (s.sessions, s.concurrency, s.turns, s.seed) == (256, 32, 6, 0)
    assert (s.first_len, s.user_len, s.gen_len) == ((2000, 8000), (200, 1000), (200, 500))
    a = bench.parse([])
    assert (a.sessions, a.concurrency, a.turns, a.seed, a.gpus) == (256, 32, 6, 0, 1)
    assert (tuple(a.first_len), tuple(a.user_len), tuple(a.gen_len)) == ((2000, 8000), (200, 1000), (200, 500))
