"""Native block bookkeeping (libpagekv pk_bm_*) against pagellm: replay of golden traces
recorded from pagellm's BlockManager, plus pagellm's own allocator tests
(tests/unit/test_paged.py:60-147) run against the native classes. CPU only."""

from __future__ import annotations

import pytest
from conftest import load_traces
from test_oracle_golden import _replay

from pagellm_b200.cache import BlockAllocator, BlockManager, OutOfBlocks, block_hash


@pytest.mark.parametrize("ti", [0, 1, 2])
def test_native_manager_replays_pagellm_trace(ti):
    """Same ops -> same return values, tables, ref counts, free-list order, LRU order and
    prefix statistics after every op, bit for bit."""
    _replay(load_traces()[ti], BlockManager, OutOfBlocks)


def test_allocator_free_list_and_refcount():
    a = BlockAllocator(3, enable_prefix_caching=False)
    b0, b1, _ = a.allocate(), a.allocate(), a.allocate()
    assert a.num_free == 0
    with pytest.raises(OutOfBlocks):
        a.allocate()
    a.incref(b1)
    a.decref(b1)
    assert a.num_free == 0
    a.decref(b1)
    assert a.num_free == 1 and a.allocate() == b1
    a.decref(b0)
    with pytest.raises(RuntimeError):
        a.decref(b0)


def test_fork_copy_on_write_copies_only_partial_block():
    bm = BlockManager(16, block_size=4)
    bm.allocate(0, list(range(10)))
    bm.fork(0, 1)
    shared = bm.block_table(0)
    assert bm.block_table(1) == shared and all(bm.alloc.ref[b] == 2 for b in shared)
    copies = bm.ensure_capacity(1, 11, write_from=10)
    assert copies == [(shared[2], bm.block_table(1)[2])]
    assert bm.block_table(1)[:2] == shared[:2]
    assert bm.alloc.ref[shared[2]] == 1
    assert bm.ensure_capacity(0, 11, write_from=10) == []


def test_prefix_cache_hit_and_reuse():
    bm = BlockManager(32, block_size=4)
    prompt = list(range(13))
    assert bm.allocate(0, prompt) == 0
    bm.mark_computed(0, prompt, 13)
    other = [*prompt[:12], 99, 98]
    assert bm.allocate(1, other) == 12
    assert bm.block_table(1)[:3] == bm.block_table(0)[:3]
    assert bm.allocate(2, prompt[:12]) == 8


def test_prefix_cache_survives_free_until_evicted():
    bm = BlockManager(4, block_size=4)
    p = list(range(9))
    bm.allocate(0, p)
    bm.mark_computed(0, p, 9)
    bm.free(0)
    assert bm.alloc.num_free == 4
    assert bm.allocate(1, p) == 8
    bm.free(1)
    bm.allocate(2, [50 + i for i in range(16)])
    assert bm.alloc.cached == {}
    bm.free(2)
    assert bm.allocate(3, p) == 0


def test_block_hash_is_position_aware():
    a = block_hash(b"", [1, 2, 3, 4])
    b = block_hash(block_hash(b"", [9, 9, 9, 9]), [1, 2, 3, 4])
    assert a != b and a == block_hash(b"", [1, 2, 3, 4])


def test_prefix_caching_disabled():
    bm = BlockManager(16, 4, enable_prefix_caching=False)
    p = list(range(9))
    bm.allocate(0, p)
    bm.mark_computed(0, p, 9)
    assert bm.allocate(1, p) == 0


def test_can_append_accounts_for_cow():
    bm = BlockManager(3, block_size=4)
    bm.allocate(0, [1, 2, 3, 4, 5, 6])
    bm.fork(0, 1)
    assert bm.can_append(1, 7)
    bm.ensure_capacity(1, 7, 6)
    assert not bm.can_append(0, 9)


def test_errors_map_to_pagellm_exceptions():
    bm = BlockManager(8, 4)
    bm.allocate(0, [1, 2, 3])
    with pytest.raises(ValueError):
        bm.allocate(0, [1])  # duplicate sequence (paged.py:190-191)
    with pytest.raises(KeyError):
        bm.free(42)  # unknown sequence: dict.pop KeyError in pagellm
    with pytest.raises(OutOfBlocks):
        bm.allocate(1, list(range(100)))
    with pytest.raises(IndexError):
        bm.alloc.decref(99)
    bm.free(0)
    assert bm.alloc.num_used == 0 and 0 not in bm.tables


def test_tables_view_and_csr():
    bm = BlockManager(64, 4)
    for s, n in enumerate((5, 9, 1)):
        bm.allocate(s, list(range(n)))
    bm.mark_computed(1, list(range(9)), 9)
    indptr, ids = bm.tables_csr([2, 0, 1])
    assert indptr.tolist() == [0, 1, 3, 6]
    assert ids.tolist() == bm.block_table(2) + bm.block_table(0) + bm.block_table(1)
    t = bm.tables[1]
    assert t.blocks == bm.block_table(1) and len(t.hashes) == 2
    assert t.hashes[1] == block_hash(t.hashes[0], list(range(4, 8)))
    assert sorted(bm.tables) == [0, 1, 2] and len(bm.tables) == 3


def test_many_blocks_fifo_and_lru_scale():
    """100k-block pool (C5 scale): FIFO reuse order and LRU eviction order hold."""
    n = 100_000
    a = BlockAllocator(n, enable_prefix_caching=True)
    got = [a.allocate() for _ in range(n)]
    assert got == list(range(n)) and a.num_free == 0
    for b in (5, 3, 9):
        a.register(b, block_hash(b"", [b]))
    for b in (9, 7, 5, 3):
        a.decref(b)
    assert a.free == [7] and list(a.evictable) == [9, 5, 3]
    assert a.allocate() == 7
    assert a.allocate() == 9  # least recently released cached block evicted first
    assert a.lookup(block_hash(b"", [9])) is None and a.lookup(block_hash(b"", [5])) == 5
