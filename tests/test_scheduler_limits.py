"""Scheduler limits on the host (fake runner): every prefill step stays within the token budget
and every segment within the prefill chunk; a prompt that cannot fit the lane's sequence limit is
refused with an error and the others are served; long prompts are cut into chunks that resume
exactly where the previous one ended (the fake runner asserts the start of every forward)."""

import random

import pytest

from fake_runner import FakeRunner, greedy
from qwen35_b200.serving.block_pool import BlockAllocator
from qwen35_b200.serving.scheduler import Request, Scheduler
from qwen35_b200.serving.session_cache import SessionCache


class RecordingRunner(FakeRunner):
    """Keeps each prefill call's segment lengths."""

    def __init__(self, **kw):
        super().__init__(**kw)
        self.prefill_steps = []

    def prefill_batch(self, calls):
        self.prefill_steps.append([len(ids) for _, ids, _ in calls])
        return super().prefill_batch(calls)

    def decode_mixed(self, lanes, tokens, positions, calls):
        self.prefill_steps.append([len(ids) for _, ids, _ in calls])
        return super().decode_mixed(lanes, tokens, positions, calls)


@pytest.mark.parametrize("chunk,budget,mixed", [(16, 40, False), (7, 7, False), (32, 64, True)])
def test_prefill_steps_respect_chunk_and_budget(chunk, budget, mixed):
    rng = random.Random(7)
    r = RecordingRunner(max_batch=4, num_snapshots=16, block_size=4)
    s = Scheduler(r, SessionCache(BlockAllocator(2000, 4), 4, 16), prefill_chunk=chunk, token_budget=budget,
                  mixed=mixed)
    outs = []
    for _ in range(6):
        prompt = [rng.randrange(1000) for _ in range(rng.randint(1, 90))]
        toks = []
        s.submit(Request(prompt, 5, lambda e, toks=toks: toks.append(e[1]) if e[0] == "tok" else None))
        outs.append((prompt, toks))
    s.run_until_idle()
    for prompt, toks in outs:
        assert toks == greedy(prompt, 5)
    assert r.prefill_steps
    for seg in r.prefill_steps:
        assert all(0 < n <= chunk for n in seg), seg
        assert sum(seg) <= budget, seg


def test_prompt_beyond_the_sequence_limit_is_refused_and_others_served():
    r = RecordingRunner(max_batch=2, num_snapshots=8, block_size=4, max_seq=64)
    s = Scheduler(r, SessionCache(BlockAllocator(400, 4), 4, 8))
    events, good = [], []
    s.submit(Request(list(range(60)), 10, events.append))  # 60 + 10 > 64
    s.submit(Request(list(range(20)), 4, lambda e: good.append(e[1]) if e[0] == "tok" else None))
    s.run_until_idle()
    assert events and events[0][0] == "error" and "exceeds" in events[0][1]
    assert good == greedy(list(range(20)), 4)
