"""Session-cache behaviour under snapshot pressure (host only): a closed-loop multi-turn
workload with few snapshot slots must still resume every follow-up turn from the previous
turn's close, so the only prompt tokens prefilled are the opening prompts and each turn's new
tokens. Snapshots held by nodes a conversation has moved past (its earlier turn-open and
turn-close nodes) are reclaimed instead of pinning the pool."""

from qwen35_b200.serving.block_pool import BlockAllocator
from qwen35_b200.serving.scheduler import Scheduler
from qwen35_b200.serving.session_cache import SessionCache
from qwen35_b200.serving.workload import ChatSpec, ClosedLoop


class CountingRunner:
    """Scheduler-facing stand-in that only counts prefilled tokens."""

    def __init__(self, max_batch, num_snapshots, block_size, max_seq):
        self.max_batch, self.num_snapshots, self.block_size, self.max_seq = max_batch, num_snapshots, block_size, max_seq
        self.prefill_tokens = 0

    def begin(self, lane): pass
    def attach_blocks(self, lane, blocks): pass
    def extend_blocks(self, grants): pass
    def copy_block(self, d, s, n): pass
    def save_snapshot(self, lane, snap): pass
    def load_snapshot(self, lane, snap): pass
    def cache_node_logits(self, snap, lg): pass
    def cached_node_logits(self, snap): return [0]
    def decode_row(self, lg, i): return [0]
    def decode_tokens_per_step(self): return 1

    def prefill_batch(self, calls):
        self.prefill_tokens += sum(len(i) for _, i, _ in calls)
        return [[0] for _ in calls]

    def decode(self, lanes, toks, poss):
        return [[0]] * len(lanes)

    def sample_batch(self, lg, temps):
        return [7] * len(temps)


class CountingLaunchRunner(CountingRunner):
    """The same, with the one-step overlap entry points."""

    def decode_launch(self, lanes, tokens, positions, src_rows, keep_rows=()):
        return ([7] * len(lanes), {i: [0] for i in keep_rows})

    def decode_collect(self, h):
        return h[0]

    def decode_kept(self, h):
        return h[1]


import pytest


@pytest.mark.parametrize("runner_cls", [CountingRunner, CountingLaunchRunner])
def test_follow_up_turns_resume_from_the_previous_close_with_few_snapshots(runner_cls):
    lanes, snaps = 6, 2 * 6 + 2
    spec = ChatSpec(sessions=24, concurrency=lanes, turns=5, first_len=(200, 600), user_len=(20, 80),
                    gen_len=(20, 60), vocab=5000, seed=3)
    r = runner_cls(lanes, snaps, 16, 8192)
    cache = SessionCache(BlockAllocator(lanes * 8192 // 16 + 1, 16), 16, snaps)
    s = Scheduler(r, cache, prefill_chunk=256, token_budget=512)
    loop = ClosedLoop(s, spec)
    loop.start()
    while loop.active:
        s.step()
        loop.pump()
    recs = loop.records
    # opening prompts in full; each later turn: the previous turn's last sampled token (never
    # forwarded) plus the new user tokens
    expect = sum(r.prompt_len for r in recs if r.turn == 0)
    by = {(r.session, r.turn): r for r in recs}
    for r in recs:
        if r.turn > 0:
            prev = by[(r.session, r.turn - 1)]
            expect += r.prompt_len - (prev.prompt_len + prev.generated - 1)
    assert all(x.error is None for x in recs)
    assert cache.admissions["hit"] == 24 * 4 and cache.admissions["miss_cold"] == 24
    assert sum(x.reused for x in recs if x.turn > 0) == sum(by[(x.session, x.turn - 1)].prompt_len
                                                           + by[(x.session, x.turn - 1)].generated - 1
                                                           for x in recs if x.turn > 0)
    assert cache.reclaims > 0
    assert loop.sched.runner.prefill_tokens == expect


def test_cache_stats_line(monkeypatch, capsys):
    monkeypatch.setenv("QB_CACHE_STATS", "2")
    r = CountingRunner(2, 6, 16, 4096)
    s = Scheduler(r, SessionCache(BlockAllocator(600, 16), 16, 6))
    loop = ClosedLoop(s, ChatSpec(sessions=2, concurrency=2, turns=2, first_len=(40, 60), user_len=(5, 9),
                                  gen_len=(3, 5), vocab=500, seed=1))
    loop.start()
    while loop.active:
        s.step()
        loop.pump()
    lines = [ln for ln in capsys.readouterr().out.splitlines() if ln.startswith("[cache-stats]")]
    assert len(lines) == 2 and "finished=4" in lines[-1] and "hit=2" in lines[-1]
