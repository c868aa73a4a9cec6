"""Paged KV block pool: a refcounted free list over block ids (host only, torch-free).

Block ``RESERVED_BLOCK`` (0) is never handed out: padded rows of captured graphs and unused
block-table entries point at it, so a masked write can never land in a live block. Every other
id carries a reference count; the scheduler's session cache takes one reference per holder
(a trie node, or a lane that borrows a node's blocks), so a block is free exactly when nobody
can still read it. Reference behaviour: ``block_pool.py:38-224``.
"""

from __future__ import annotations

from collections import deque
from collections.abc import Iterable

RESERVED_BLOCK = 0


class PoolExhausted(RuntimeError):
    pass


class BlockAllocator:
    def __init__(self, num_blocks: int, block_size: int) -> None:
        if num_blocks < 2:
            raise ValueError("need at least one usable block besides the reserved one")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self._free: deque[int] = deque(range(1, num_blocks))
        self._ref = [0] * num_blocks

    def free_count(self) -> int:
        return len(self._free)

    def usable_blocks(self) -> int:
        return self.num_blocks - 1

    def capacity_tokens(self) -> int:
        return self.usable_blocks() * self.block_size

    def alloc(self, n: int) -> list[int]:
        """``n`` fresh ids with refcount 1 (all or nothing)."""
        if n < 0:
            raise ValueError("negative allocation")
        if n > len(self._free):
            raise PoolExhausted(f"requested {n} blocks, {len(self._free)} free")
        out = [self._free.popleft() for _ in range(n)]
        for b in out:
            self._ref[b] = 1
        return out

    def incref(self, ids: Iterable[int]) -> None:
        for b in ids:
            self._check(b, "incref")
            self._ref[b] += 1

    def decref(self, ids: Iterable[int]) -> None:
        for b in ids:
            self._check(b, "decref")
            self._ref[b] -= 1
            if self._ref[b] == 0:
                self._free.append(b)

    def refcount(self, b: int) -> int:
        return self._ref[b]

    def _check(self, b: int, op: str) -> None:
        if b == RESERVED_BLOCK:
            raise ValueError(f"{op} of the reserved block")
        if not (0 < b < self.num_blocks):
            raise ValueError(f"{op} of out-of-range block {b}")
        if self._ref[b] <= 0:
            raise ValueError(f"{op} of free block {b}")


def blocks_for(tokens: int, block_size: int) -> int:
    return (tokens + block_size - 1) // block_size


def physical_row(table: list[int], pos: int, block_size: int) -> int:
    return table[pos // block_size] * block_size + pos % block_size


def padded_row(table: list[int], max_blocks: int) -> list[int]:
    return list(table) + [RESERVED_BLOCK] * (max_blocks - len(table))
