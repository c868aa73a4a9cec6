from qwen35_b200.serving.block_pool import BlockAllocator
from qwen35_b200.serving.session_cache import SessionCache


def mk(blocks=64, bs=4, snaps=4):
    return SessionCache(BlockAllocator(blocks, bs), bs, snaps)


def test_lookup_publish_and_refs():
    c = mk()
    blocks = c.reserve_blocks(3)
    toks = list(range(10))
    s = c.reserve_snapshot()
    n = c.publish(toks, 10, blocks, s)
    assert c.lookup(toks + [99]) is n
    assert c.lookup([5] + toks).is_root()
    assert all(c.alloc.refcount(b) == 2 for b in blocks)  # lane + node
    c.release_lane_blocks(blocks)
    assert all(c.alloc.refcount(b) == 1 for b in blocks)


def test_cow_needed_for_partial_last_block():
    c = mk()
    b = c.reserve_blocks(3)
    n = c.publish(list(range(10)), 10, b, c.reserve_snapshot())
    assert c.needs_cow(n)
    new = c.reserve_blocks(1)
    lane = c.adopt(n, new[0])
    assert lane[:-1] == b[:-1] and lane[-1] == new[0]


def test_lru_leaf_eviction_frees_blocks():
    c = mk(blocks=9, bs=4, snaps=8)
    b1 = c.reserve_blocks(4)
    n1 = c.publish(list(range(16)), 16, b1, c.reserve_snapshot())
    c.release_lane_blocks(b1)
    b2 = c.reserve_blocks(4)
    c.publish([7] * 16, 16, b2, c.reserve_snapshot())
    c.release_lane_blocks(b2)
    got = c.reserve_blocks(4)  # forces eviction of the LRU leaf (n1)
    assert len(got) == 4 and c.lookup(list(range(16)) + [1]).is_root()
    assert c.node_count() == 1 and n1.parent is not None


def test_snapshot_reclaim_prefers_superseded_internal():
    c = mk(blocks=64, bs=4, snaps=2)
    t1 = list(range(8))
    b = c.reserve_blocks(2)
    n1 = c.publish(t1, 8, b, c.reserve_snapshot())
    lane = c.adopt(n1)
    b2 = lane + c.reserve_blocks(1)
    n2 = c.publish(t1 + [50, 51, 52, 53], 12, b2, c.reserve_snapshot(), resumed_from=n1)
    assert n1.superseded and n2.parent is n1
    s = c.reserve_snapshot()  # pool full -> reclaims n1's snapshot, keeps n2
    assert n1.snapshot == -1 and n2.snapshot >= 0 and s >= 0
    assert c.lookup(t1 + [50, 51, 52, 53, 9]) is n2
    assert c.lookup(t1 + [1]).is_root()


def test_evict_all_respects_protect():
    c = mk()
    b = c.reserve_blocks(2)
    n = c.publish(list(range(8)), 8, b, c.reserve_snapshot())
    b2 = c.reserve_blocks(2)
    c.publish([3] * 8, 8, b2, c.reserve_snapshot())
    assert c.evict_all(protect=[n]) == 1
    assert c.node_count() == 1


def test_classify_cold_hit_evicted_reclaimed():
    c = mk(blocks=12, bs=4, snaps=8)
    p1 = list(range(100, 120))
    assert c.classify(p1, c.lookup(p1)) == "miss_cold"
    b = c.reserve_blocks(5)
    c.publish(p1, 20, b, c.reserve_snapshot())
    c.release_lane_blocks(b)
    assert c.classify(p1 + [1, 2], c.lookup(p1 + [1, 2])) == "hit"
    assert c.classify(p1, c.lookup(p1)) == "exact"
    c.evict_all()
    assert c.classify(p1 + [1], c.lookup(p1 + [1])) == "miss_evicted"
    assert c.classify(list(range(300, 330)), c.root) == "miss_cold"
    # a deeper boundary whose snapshot was reclaimed
    b = c.reserve_blocks(5)
    n = c.publish(p1, 20, b, c.reserve_snapshot())
    c.release_lane_blocks(b)
    c.release_snapshot(n.snapshot)
    n.snapshot, n.reclaimed = -1, True  # as _reclaim_one_internal leaves a node
    assert c.classify(p1 + [3], c.lookup(p1 + [3])) == "miss_reclaimed"
    assert c.admissions["miss_cold"] == 2 and c.admissions["hit"] == 1


def test_classify_remembers_each_evicted_session_sharing_a_prefix():
    """Two sessions with the same first 20 tokens lose boundaries at the same depth: both are
    reported as evicted, not only the last one evicted."""
    c = mk(blocks=40, bs=4, snaps=8)
    shared = list(range(500, 520))
    a, b = shared + [1] * 8, shared + [2] * 8
    for p in (a, b):
        blk = c.reserve_blocks(7)
        c.publish(p, 28, blk, c.reserve_snapshot())
        c.release_lane_blocks(blk)
    c.evict_all()
    for p in (a, b):
        assert c.classify(p + [7], c.lookup(p + [7])) == "miss_evicted"
    assert c.classify(shared + [3] * 8, c.root) == "miss_cold"
    # the memo of the last lookup is used only for that same prompt object
    q = a + [9]
    node = c.lookup(q)
    assert c._lookup_memo[0] is q and c.classify(q, node) == "miss_evicted"


def test_prefix_digests_match_per_prefix():
    from qwen35_b200.serving.session_cache import SessionCache

    toks = [5, 0, 7, 7, 123456, 3]
    all_d = SessionCache._prefix_digests(toks, range(1, 7))
    for d in range(1, 7):
        assert SessionCache._prefix_digests(toks[:d], [d])[d] == all_d[d]
    assert len(set(all_d.values())) == 6
    assert SessionCache._prefix_digests(toks, [0, 9]) == {}
