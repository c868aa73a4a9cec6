"""Tensor/expert-parallel sharding arithmetic (pure Python, no torch).

Megatron column -> row convention: every projection that feeds a per-head or per-expert
computation is split by output rows (column parallel); the projection back to the hidden size
is split by input columns (row parallel) and its partial sums are all-reduced. Reference
behaviour: ``tp.py:130-214`` (``Shard``, ``even``, ``kv_shard``, ``Plan``, ``plan``) and
``deltanet_tp.py:1-159``.

* Attention: query heads split evenly. When there are fewer KV heads than ranks each KV head
  is replicated on ``world / kv_heads`` consecutive ranks; query head ``h`` always reads KV
  head ``h // (q_heads / kv_heads)``, which this plan keeps on the same rank.
* Gated DeltaNet: key heads and value heads split evenly. Value head ``h`` reads key head
  ``h // (v_heads / k_heads)``; with both split evenly, rank ``r``'s value heads read only
  rank ``r``'s key heads, so the recurrence is block diagonal over ranks and needs no
  communication.
* MoE: whole experts per rank (expert parallel); the shared expert's intermediate is split.
* LM head: vocabulary rows split (vocab parallel).
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    start: int
    stop: int

    @property
    def count(self) -> int:
        return self.stop - self.start

    def slice(self) -> slice:
        return slice(self.start, self.stop)


def even(total: int, rank: int, world: int, what: str = "dim") -> Shard:
    if total % world:
        raise ValueError(f"{what}={total} does not split evenly over {world} ranks")
    n = total // world
    return Shard(rank * n, (rank + 1) * n)


@dataclass(frozen=True)
class KVShard(Shard):
    replicas: int  # ranks holding each KV head (1 when heads are split, not replicated)


def kv_shard(kv_heads: int, rank: int, world: int) -> KVShard:
    if kv_heads >= world:
        s = even(kv_heads, rank, world, "kv_heads")
        return KVShard(s.start, s.stop, 1)
    if world % kv_heads:
        raise ValueError(f"world={world} is not a multiple of kv_heads={kv_heads}")
    rep = world // kv_heads
    h = rank // rep
    return KVShard(h, h + 1, rep)


@dataclass(frozen=True)
class Plan:
    rank: int
    world: int
    q: Shard
    kv: KVShard
    dn_k: Shard
    dn_v: Shard
    experts: Shard
    shared: Shard
    vocab: Shard

    @property
    def ep(self) -> int:
        return self.world


def plan(cfg, rank: int, world: int, vocab_parallel: bool = True) -> Plan:
    q = even(cfg.q_heads, rank, world, "q_heads")
    kv = kv_shard(cfg.kv_heads, rank, world)
    group = cfg.q_heads // cfg.kv_heads
    for h in (q.start, q.stop - 1):
        if not (kv.start <= h // group < kv.stop):
            raise ValueError(f"rank {rank}: q head {h} reads kv head {h // group} outside {kv}")
    dn_k = even(cfg.dn_k_heads, rank, world, "dn_k_heads")
    dn_v = even(cfg.dn_v_heads, rank, world, "dn_v_heads")
    experts = even(cfg.experts, rank, world, "experts")
    shared = even(cfg.shared_inter, rank, world, "shared_inter")
    vocab = even(cfg.vocab, rank, world, "vocab") if vocab_parallel else Shard(0, cfg.vocab)
    return Plan(rank, world, q, kv, dn_k, dn_v, experts, shared, vocab)
