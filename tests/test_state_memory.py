"""Long-run memory invariants (host only): 12 sessions x 20 turns through the real scheduler,
block pool and session cache on tight pools (eviction and snapshot reclaim all the time). While
it runs, every block is either free or referenced; at the end, once the cache is emptied, every
block and every snapshot slot is free again and only the trie root is left: nothing leaks."""

import random

from fake_runner import FakeRunner, greedy
from qwen35_b200.serving.block_pool import BlockAllocator
from qwen35_b200.serving.scheduler import Request, Scheduler
from qwen35_b200.serving.session_cache import SessionCache


def test_no_block_or_snapshot_leaks_over_many_turns():
    blocks, snaps, bs = 400, 24, 4
    alloc = BlockAllocator(blocks, bs)
    cache = SessionCache(alloc, bs, snaps)
    r = FakeRunner(max_batch=4, num_snapshots=snaps, block_size=bs)
    s = Scheduler(r, cache)
    rng = random.Random(0)
    hist = {k: [rng.randrange(900) for _ in range(rng.randint(5, 30))] for k in range(12)}
    for turn in range(20):
        res = {}
        for k in range(12):
            toks, ends = [], []
            res[k] = (list(hist[k]), toks, ends)
            s.submit(Request(list(hist[k]), 6,
                             lambda e, toks=toks, ends=ends: toks.append(e[1]) if e[0] == "tok" else ends.append(e)))
        s.run_until_idle()
        for k in range(12):
            prompt, toks, ends = res[k]
            assert ends and ends[-1][0] == "end", ends
            assert toks == greedy(prompt, 6)  # the cache never changed an answer
            hist[k] = (prompt + toks + [rng.randrange(900) for _ in range(rng.randint(3, 12))])[-120:]
        # every block is free or referenced by someone (no block lost between the two)
        used = sum(1 for b in range(1, blocks) if alloc.refcount(b) > 0)
        assert used + alloc.free_count() == blocks - 1
    assert len(s.free_lanes) == 4
    st = cache.stats()
    assert st.evictions > 0 and st.hits > 0  # the pools were tight and the cache was used
    assert sum(st.admissions.values()) == 12 * 20 and st.admissions.get("miss_cold", 0) >= 12
    cache.evict_all()
    assert alloc.free_count() == blocks - 1
    assert cache.free_snapshot_count() == snaps
    assert not cache.root.children
