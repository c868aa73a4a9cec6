import pytest

from qwen35_b200.serving.block_pool import RESERVED_BLOCK, BlockAllocator, PoolExhausted, blocks_for, physical_row


def test_reserved_block_never_allocated():
    a = BlockAllocator(5, 16)
    got = a.alloc(4)
    assert RESERVED_BLOCK not in got and sorted(got) == [1, 2, 3, 4]
    with pytest.raises(PoolExhausted):
        a.alloc(1)


def test_refcount_free_cycle():
    a = BlockAllocator(4, 16)
    b = a.alloc(2)
    a.incref(b)
    a.decref(b)
    assert a.free_count() == 1
    a.decref(b)
    assert a.free_count() == 3
    with pytest.raises(ValueError):
        a.decref([b[0]])


def test_reserved_and_range_checks():
    a = BlockAllocator(4, 16)
    with pytest.raises(ValueError):
        a.incref([0])
    with pytest.raises(ValueError):
        a.incref([9])


def test_all_or_nothing():
    a = BlockAllocator(3, 16)
    with pytest.raises(PoolExhausted):
        a.alloc(3)
    assert a.free_count() == 2


def test_row_arithmetic():
    assert blocks_for(0, 16) == 0 and blocks_for(16, 16) == 1 and blocks_for(17, 16) == 2
    assert physical_row([5, 9], 17, 16) == 9 * 16 + 1
