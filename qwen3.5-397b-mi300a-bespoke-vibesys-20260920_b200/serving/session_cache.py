"""Cross-turn prefix / session cache: a trie of snapshot boundaries (host only, torch-free).

A ``Node`` is a token prefix at which some request's state was recorded: its paged KV blocks
(refcounted in the shared ``BlockAllocator``) and one snapshot slot of the runner's DeltaNet
conv + recurrent state pool (plus the cached next-token logits of that prefix). Nodes exist
only at boundaries (turn open / turn close), because a recurrent state exists only where one
was saved; the trie branches at nodes, and two children of one node may share a prefix of
their edges.

* ``Node.blocks`` is the complete flat block list for ``[0, depth)``; each id holds one
  reference on the node's behalf. A lane resuming from a node takes its own references
  (``adopt``), so evicting the node can never free blocks a live lane still reads.
* Copy-on-write: when ``depth`` is not a multiple of the block size the node's last block is
  partial; a second writer must copy it first (``needs_cow``; the caller does the device copy).
* Eviction: LRU over leaves only (an internal node's blocks are part of its descendants'
  context). Before evicting any leaf, ``reserve_snapshot`` reclaims the snapshot slot of the
  least recently used *superseded* internal node: one that a request resumed from and then
  published a deeper node under, so its conversation has provably moved past it. The node
  keeps its blocks and trie position (``snapshot = -1``); ``lookup`` skips stateless nodes.

Reference behaviour: ``session_cache.py:1-614`` (``Node``, ``SessionCache.lookup_detail``,
``needs_cow``, ``adopt``, ``reserve_blocks``, ``reserve_snapshot``, ``publish``,
``_reclaim_one_internal``, ``evict_all``).
"""

from __future__ import annotations

import itertools
from collections import Counter, OrderedDict
from collections.abc import Sequence
from dataclasses import dataclass, field

from .block_pool import BlockAllocator, PoolExhausted, blocks_for


class SessionCacheError(RuntimeError):
    """Nothing left to evict for an admission."""


@dataclass(eq=False)
class Node:
    parent: Node | None
    edge: tuple[int, ...]
    depth: int
    blocks: tuple[int, ...]
    snapshot: int
    children: dict[int, list[Node]] = field(default_factory=dict)
    used: int = 0
    reclaimed: bool = False  # its snapshot was taken back to free a slot
    adopted: bool = False
    superseded: bool = False

    def is_leaf(self) -> bool:
        return not self.children

    def is_root(self) -> bool:
        return self.parent is None

    def has_state(self) -> bool:
        return self.parent is None or self.snapshot >= 0


@dataclass(frozen=True)
class CacheStats:
    nodes: int
    snapshots_used: int
    snapshots_capacity: int
    free_blocks: int
    evictions: int
    reclaims: int
    hits: int
    misses: int
    admissions: dict = field(default_factory=dict)  # classify() counts


class SessionCache:
    def __init__(self, allocator: BlockAllocator, block_size: int, num_snapshots: int) -> None:
        self.alloc = allocator
        self.block_size = block_size
        self.num_snapshots = num_snapshots
        self.root = Node(None, (), 0, (), -1)
        self._free_snaps = list(range(num_snapshots - 1, -1, -1))
        self._clock = itertools.count(1)
        self.evictions = 0
        self.reclaims = 0
        self.hits = 0
        self.misses = 0
        self.admissions: Counter = Counter()  # classify() results
        self._evicted: OrderedDict = OrderedDict()  # (first tokens, depth, digest) of evicted boundaries, LRU
        self._evicted_by_key: dict[tuple, dict[int, set]] = {}  # first tokens -> depth -> prefix digests
        self._lookup_memo: tuple | None = None  # (prompt, node, deepest reclaimed depth) of the last lookup

    # ------------------------------------------------------------------ lookup
    def _walk(self, prompt: Sequence[int]):
        """Yield the nodes along ``prompt`` from the root, deepest last."""
        node = self.root
        yield node
        while True:
            nxt = None
            if node.depth < len(prompt):
                for c in node.children.get(prompt[node.depth], ()):
                    if c.depth <= len(prompt) and tuple(prompt[node.depth:c.depth]) == c.edge:
                        if nxt is None or c.depth > nxt.depth:
                            nxt = c
            if nxt is None:
                return
            node = nxt
            yield node

    def lookup(self, prompt: Sequence[int]) -> Node:
        """Deepest node with a resumable state whose span is a prefix of ``prompt``. The same
        walk notes the deepest matching boundary whose snapshot was reclaimed, which
        ``classify`` reuses instead of walking again."""
        best, reclaimed = self.root, -1
        for n in self._walk(prompt):
            if n.has_state():
                best = n
            elif n.reclaimed:
                reclaimed = n.depth
        self._lookup_memo = (prompt, best, reclaimed)
        if best.is_root():
            self.misses += 1
        else:
            self.hits += 1
            self._touch(best)
        return best

    def deepest(self, prompt: Sequence[int]) -> Node:
        """Deepest node (with or without state) along ``prompt``."""
        last = self.root
        for n in self._walk(prompt):
            last = n
        return last

    EVICTED_INDEX = 4096  # remembered evicted boundaries (diagnostics only)
    EVICTED_KEY = 16  # leading tokens that bucket them

    @staticmethod
    def _prefix_digests(tokens: Sequence[int], depths) -> dict[int, int]:
        """Digest of ``tokens[:d]`` for each ``d`` in ``depths``: a polynomial hash mod 2^64
        computed for every prefix in one vectorised pass (one walk of the longest prefix,
        however many depths are asked)."""
        import numpy as np

        depths = [d for d in depths if 0 < d <= len(tokens)]
        if not depths:
            return {}
        n = max(depths)
        t = np.asarray(tokens[:n], dtype=np.uint64) + np.uint64(1)
        powers = np.cumprod(np.full(n, 1_000_003, dtype=np.uint64), dtype=np.uint64)
        with np.errstate(over="ignore"):
            cs = np.cumsum(t * powers, dtype=np.uint64)
        return {d: int(cs[d - 1]) for d in depths}

    def _note_evicted(self, node: Node) -> None:
        """Remember that a boundary with state at ``node`` was evicted (for ``classify``). Several
        sessions that share their first tokens may lose boundaries at the same depth: each
        keeps its own digest."""
        edges = []
        n = node
        while n is not None and not n.is_root():
            edges.append(n.edge)
            n = n.parent
        path = tuple(t for e in reversed(edges) for t in e)
        if len(path) < self.EVICTED_KEY:
            return
        digest = self._prefix_digests(path, [len(path)])[len(path)]
        ent = (path[: self.EVICTED_KEY], node.depth, digest)
        self._evicted[ent] = None
        self._evicted.move_to_end(ent)
        self._evicted_by_key.setdefault(ent[0], {}).setdefault(node.depth, set()).add(digest)
        while len(self._evicted) > self.EVICTED_INDEX:
            (k, d, dg), _ = self._evicted.popitem(last=False)
            by_depth = self._evicted_by_key[k]
            by_depth[d].discard(dg)
            if not by_depth[d]:
                del by_depth[d]
            if not by_depth:
                del self._evicted_by_key[k]

    def classify(self, prompt: Sequence[int], node: Node) -> str:
        """Why an admission of ``prompt`` resumes at ``node`` (from ``lookup``), for the cache
        statistics: ``exact`` / ``hit`` (nothing deeper was cached that this cache remembers),
        ``short_reclaimed`` / ``miss_reclaimed`` (a deeper boundary matches but its snapshot was
        reclaimed), ``short_evicted`` / ``miss_evicted`` (a deeper boundary matching the prompt
        was evicted), ``miss_cold`` (nothing matches, now or before). Reference behaviour:
        ``session_cache.py:209-227`` (``classify``)."""
        kind = "miss" if node.is_root() else "short"
        memo = self._lookup_memo
        if memo is not None and memo[0] is prompt and memo[1] is node:
            reclaimed = memo[2]
        else:
            reclaimed = max((n.depth for n in self._walk(prompt) if n.reclaimed), default=-1)
        if reclaimed > node.depth:
            cls = kind + "_reclaimed"
        else:
            cls = None
            by_depth = self._evicted_by_key.get(tuple(prompt[: self.EVICTED_KEY]), {})
            cand = [d for d in by_depth if node.depth < d <= len(prompt)]
            if cand:
                got = self._prefix_digests(prompt, cand)
                if any(got[d] in by_depth[d] for d in cand):
                    cls = kind + "_evicted"
            if cls is None:
                cls = "miss_cold" if node.is_root() else ("exact" if node.depth == len(prompt) else "hit")
        self.admissions[cls] += 1
        return cls

    # ------------------------------------------------------------------ adoption
    def needs_cow(self, node: Node) -> bool:
        return node.depth % self.block_size != 0 and not node.is_root()

    def adopt(self, node: Node, replacement_last_block: int | None = None) -> list[int]:
        """A lane starts from ``node``: returns its block list with one new reference per id
        (the replacement block, from ``reserve_blocks``, already holds its reference)."""
        blocks = list(node.blocks)
        if replacement_last_block is not None:
            blocks[-1] = replacement_last_block
            self.alloc.incref(blocks[:-1])
        else:
            self.alloc.incref(blocks)
        if not node.is_root():
            node.adopted = True
            self._touch(node)
        return blocks

    def release_lane_blocks(self, blocks: Sequence[int]) -> None:
        self.alloc.decref(blocks)

    # ------------------------------------------------------------------ reservation
    def reserve_blocks(self, n: int, protect: Sequence[Node] = ()) -> list[int]:
        while self.alloc.free_count() < n:
            if not self._evict_one_leaf(protect):
                raise SessionCacheError(f"KV block pool exhausted: need {n}, free {self.alloc.free_count()}")
        try:
            return self.alloc.alloc(n)
        except PoolExhausted as e:  # pragma: no cover - guarded by the loop above
            raise SessionCacheError(str(e)) from e

    def reserve_snapshot(self, protect: Sequence[Node] = ()) -> int:
        if self._free_snaps:
            return self._free_snaps.pop()
        if self._reclaim_one_internal(protect) or self._evict_one_leaf(protect, need_snapshot=True):
            if self._free_snaps:
                return self._free_snaps.pop()
        raise SessionCacheError("snapshot pool exhausted")

    def release_snapshot(self, snap: int) -> None:
        self._free_snaps.append(snap)

    # ------------------------------------------------------------------ publishing
    def publish(self, tokens: Sequence[int], depth: int, blocks: Sequence[int], snapshot: int,
                resumed_from: Node | None = None) -> Node:
        """Record the boundary ``tokens[:depth]`` with the lane's ``blocks`` (refs are taken here)
        and the already-saved ``snapshot``. If an identical node exists, the new snapshot is
        released (or adopted when the node had lost its own) and the existing node returned."""
        span = tuple(tokens[:depth])
        parent = self.root
        for n in self._walk(span):
            parent = n
        nb = blocks_for(depth, self.block_size)
        if parent.depth == depth and not parent.is_root():
            if parent.snapshot < 0:
                parent.snapshot, parent.reclaimed = snapshot, False
            else:
                self.release_snapshot(snapshot)
            self._touch(parent)
            return parent
        node = Node(parent, span[parent.depth:], depth, tuple(blocks[:nb]), snapshot)
        self.alloc.incref(node.blocks)
        parent.children.setdefault(node.edge[0], []).append(node)
        self._touch(node)
        if resumed_from is not None and not resumed_from.is_root() and resumed_from is not node:
            a = node.parent
            while a is not None and a is not resumed_from:
                a = a.parent
            if a is resumed_from:
                resumed_from.superseded = True
        return node

    # ------------------------------------------------------------------ eviction
    def _protected(self, protect: Sequence[Node]) -> set[int]:
        s = set()
        for p in protect:
            while p is not None:
                s.add(id(p))
                p = p.parent
        return s

    def _iter(self, node: Node | None = None):
        stack = [node or self.root]
        while stack:
            n = stack.pop()
            yield n
            for lst in n.children.values():
                stack.extend(lst)

    def _evict_one_leaf(self, protect: Sequence[Node] = (), need_snapshot: bool = False) -> bool:
        prot = self._protected(protect)
        cands = [n for n in self._iter() if n.is_leaf() and not n.is_root() and id(n) not in prot
                 and (not need_snapshot or n.snapshot >= 0)]
        if not cands:
            return False
        victim = min(cands, key=lambda n: n.used)
        self._remove(victim)
        self.evictions += 1
        return True

    def _reclaim_one_internal(self, protect: Sequence[Node] = ()) -> bool:
        """Take the snapshot slot of one internal node (superseded ones first, then any, least
        recently used first). Only the nodes in ``protect`` themselves are spared: an internal
        node's blocks are part of its descendants' context, but its snapshot is needed only by
        an admission that resumes exactly there, and a live lane already loaded its own."""
        prot = {id(p) for p in protect}
        cands = [n for n in self._iter() if not n.is_leaf() and not n.is_root() and n.snapshot >= 0
                 and n.superseded and id(n) not in prot]
        if not cands:
            cands = [n for n in self._iter() if not n.is_leaf() and not n.is_root() and n.snapshot >= 0
                     and id(n) not in prot]
        if not cands:
            return False
        victim = min(cands, key=lambda n: n.used)
        self.release_snapshot(victim.snapshot)
        victim.snapshot = -1
        victim.reclaimed = True
        self.reclaims += 1
        return True

    def _remove(self, node: Node) -> None:
        while node is not None and not node.is_root() and node.is_leaf():
            parent = node.parent
            lst = parent.children[node.edge[0]]
            lst.remove(node)
            if not lst:
                del parent.children[node.edge[0]]
            self.alloc.decref(node.blocks)
            if node.snapshot >= 0:
                self._note_evicted(node)
                self.release_snapshot(node.snapshot)
            node = parent if (parent is not None and not parent.is_root() and parent.snapshot < 0) else None

    def evict_all(self, protect: Sequence[Node] = ()) -> int:
        n = 0
        while self._evict_one_leaf(protect):
            n += 1
        return n

    def _touch(self, node: Node) -> None:
        node.used = next(self._clock)

    # ------------------------------------------------------------------ stats
    def node_count(self) -> int:
        return sum(1 for _ in self._iter()) - 1

    def free_snapshot_count(self) -> int:
        return len(self._free_snaps)

    def stats(self) -> CacheStats:
        return CacheStats(self.node_count(), self.num_snapshots - len(self._free_snaps), self.num_snapshots,
                          self.alloc.free_count(), self.evictions, self.reclaims, self.hits, self.misses,
                          dict(self.admissions))
