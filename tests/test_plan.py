"""Tensor / expert parallel sharding of the full geometry at 1, 2, 4 and 8 ranks (no GPU): every
dimension splits into disjoint, covering, equal ranges in rank order; the 2 KV heads are
replicated once the ranks outnumber them and every rank's query heads read its own KV head;
DeltaNet value heads stay with their key head's group; the tiny model splits at the widths its
heads allow and refuses the others."""

import pytest

from qwen35_b200.models.config import full_config, tiny_config
from qwen35_b200.parallel.plan import kv_shard, plan


def _covers(shards, total):
    assert [s.start for s in shards] == sorted(s.start for s in shards)
    pos = 0
    for s in shards:
        assert s.start == pos and s.count == total // len(shards)
        pos = s.stop
    assert pos == total


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_full_geometry_shards(world):
    cfg = full_config()
    ps = [plan(cfg, r, world) for r in range(world)]
    for dim, total in (("q", cfg.q_heads), ("dn_k", cfg.dn_k_heads), ("dn_v", cfg.dn_v_heads),
                       ("experts", cfg.experts), ("shared", cfg.shared_inter), ("vocab", cfg.vocab)):
        _covers([getattr(p, dim) for p in ps], total)
    group = cfg.q_heads // cfg.kv_heads
    for p in ps:
        assert p.ep == world
        for h in range(p.q.start, p.q.stop):  # GQA: the query heads read a KV head this rank holds
            assert p.kv.start <= h // group < p.kv.stop
        # DeltaNet: the value heads of a key head stay on the rank holding that key head
        per_k = cfg.dn_v_heads // cfg.dn_k_heads
        assert p.dn_v.start == p.dn_k.start * per_k and p.dn_v.stop == p.dn_k.stop * per_k
    if world > cfg.kv_heads:
        assert all(p.kv.count == 1 and p.kv.replicas == world // cfg.kv_heads for p in ps)
    else:
        _covers([p.kv for p in ps], cfg.kv_heads)
    if world == 8:  # one rank of 8: 4 query heads, 1 KV head, 2 key / 8 value DeltaNet heads, 64 experts
        p = ps[3]
        assert (p.q.count, p.kv.count, p.dn_k.count, p.dn_v.count, p.experts.count) == (4, 1, 2, 8, 64)
        assert p.shared.count == cfg.shared_inter // 8 and p.vocab.count == cfg.vocab // 8


def test_kv_replication_and_limits():
    assert [(s.start, s.replicas) for s in (kv_shard(2, r, 8) for r in range(8))] == \
        [(0, 4)] * 4 + [(1, 4)] * 4
    assert kv_shard(4, 1, 2).start == 2 and kv_shard(4, 1, 2).replicas == 1
    with pytest.raises(ValueError):
        kv_shard(2, 0, 3)  # 3 ranks cannot replicate 2 heads evenly


def test_tiny_model_splits_where_its_heads_allow():
    cfg = tiny_config()
    for world in (1, 2, 4):
        ps = [plan(cfg, r, world) for r in range(world)]
        _covers([p.experts for p in ps], cfg.experts)
    with pytest.raises(ValueError):
        plan(cfg, 0, 8)  # 4 DeltaNet key heads do not split over 8 ranks
    p = plan(cfg, 1, 4, vocab_parallel=False)
    assert (p.vocab.start, p.vocab.stop) == (0, cfg.vocab)
