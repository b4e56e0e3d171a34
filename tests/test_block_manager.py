"""Native block bookkeeping (libpagekv pk_bm_*) against pagellm: replay of golden traces
recorded from pagellm's BlockManager, plus pagellm's own allocator tests
(tests/unit/test_paged.py:60-147) run against the native classes. CPU only."""

from __future__ import annotations

import numpy as np
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


# ------------------------------------------------------------------ paged rollback (truncate)
def test_truncate_releases_tail_last_first_and_trims_chain():
    bm = BlockManager(16, block_size=4)
    toks = list(range(14))
    bm.allocate(0, toks)
    bm.mark_computed(0, toks, 14)
    blocks = bm.block_table(0)
    assert len(blocks) == 4 and len(bm.tables[0].hashes) == 3
    free_before = list(bm.alloc.free)
    bm.truncate(0, 6)  # keep blocks 0, 1 (block 1 now partial)
    assert bm.block_table(0) == blocks[:2]
    assert len(bm.tables[0].hashes) == 1
    # block 3 was never published -> free list; block 2 was -> LRU (its content still
    # matches its hash); both released last block first
    assert list(bm.alloc.free) == free_before + [blocks[3]]
    assert list(bm.alloc.evictable) == [blocks[2]]
    # block 1 was published but is partial now and private: unpublished
    assert blocks[1] not in bm.alloc.block_hash and blocks[0] in bm.alloc.block_hash


def test_truncate_keeps_shared_partial_block_published_and_cows_it_on_write():
    bm = BlockManager(16, block_size=4)
    toks = list(range(12))
    bm.allocate(0, toks)
    bm.mark_computed(0, toks, 12)
    bm.fork(0, 1)
    shared = bm.block_table(0)
    bm.truncate(1, 10)  # fork 1 rejects its last 2 tokens; block 2 is still shared
    assert bm.block_table(1) == shared and shared[2] in bm.alloc.block_hash
    copies = bm.ensure_capacity(1, 11, write_from=10)
    assert copies == [(shared[2], bm.block_table(1)[2])]
    assert bm.alloc.ref[shared[2]] == 1 and shared[2] in bm.alloc.block_hash
    assert len(bm.tables[1].hashes) == 2


def test_truncate_bounds_and_unknown_sequence():
    bm = BlockManager(8, 4)
    bm.allocate(0, [1, 2, 3, 4, 5])
    with pytest.raises(ValueError):
        bm.truncate(0, 9)  # 2 blocks hold at most 8 tokens
    with pytest.raises(ValueError):
        bm.truncate(0, -1)
    with pytest.raises(KeyError):
        bm.truncate(7, 0)
    bm.truncate(0, 8)  # no-op: capacity
    bm.truncate(0, 0)
    assert bm.block_table(0) == [] and bm.alloc.num_used == 0


def test_speculative_rollback_flow():
    """Draft k tokens, verify, keep the accepted ones, continue: the table always holds
    exactly the blocks the kept tokens need, and every write lands in a private block."""
    bm = BlockManager(64, block_size=4)
    toks = list(range(10))
    bm.allocate(0, toks)
    bm.mark_computed(0, toks, 10)
    n = 10
    rng = np.random.default_rng(3)
    for _ in range(30):
        k = int(rng.integers(1, 7))
        assert bm.can_append(0, n + k)
        bm.ensure_capacity(0, n + k, write_from=n)
        acc = int(rng.integers(0, k + 1))
        toks = toks[:n] + [int(x) for x in rng.integers(0, 50, acc)]
        n += acc
        bm.truncate(0, n)
        bm.mark_computed(0, toks, n)
        assert len(bm.block_table(0)) == bm.blocks_needed(n)
        assert len(bm.tables[0].hashes) == n // 4
        assert all(bm.alloc.ref[b] == 1 for b in bm.block_table(0))


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
def test_random_ops_with_truncate_match_oracle(seed):
    """Random allocate / grow / fork / truncate / free on the native manager and on the
    oracle restatement: identical results and state after every op."""
    from oracle import paged_oracle as po

    rng = np.random.default_rng(seed)
    nb, bs = 48, 4
    nat, ora = BlockManager(nb, bs), po.OracleBlockManager(nb, bs)
    toks: dict[int, list[int]] = {}
    base = [int(x) for x in rng.integers(0, 5, 40)]  # shared prompt material -> prefix hits
    next_id = 0
    for step in range(400):
        op = rng.choice(["alloc", "grow", "fork", "trunc", "free"], p=[0.25, 0.3, 0.1, 0.25, 0.1])
        live = sorted(toks)
        if op == "alloc" or not live:
            n = int(rng.integers(1, 30))
            t = base[:n] if rng.random() < 0.5 else [int(x) for x in rng.integers(0, 5, n)]
            res = []
            for bm, exc in ((nat, OutOfBlocks), (ora, po.OracleOutOfBlocks)):
                try:
                    res.append(bm.allocate(next_id, t))
                    bm.mark_computed(next_id, t, len(t))
                except exc:
                    res.append("oob")
            assert res[0] == res[1], step
            if res[0] != "oob":
                toks[next_id] = t
            next_id += 1
        else:
            s = int(rng.choice(live))
            t = toks[s]
            if op == "grow":
                k = int(rng.integers(1, 9))
                ok = [bool(bm.can_append(s, len(t) + k)) for bm in (nat, ora)]
                assert ok[0] == ok[1], step
                if ok[0]:
                    pairs = [[tuple(p) for p in bm.ensure_capacity(s, len(t) + k, len(t))] for bm in (nat, ora)]
                    assert pairs[0] == pairs[1], step
                    t = t + [int(x) for x in rng.integers(0, 5, k)]
                    toks[s] = t
                    for bm in (nat, ora):
                        bm.mark_computed(s, t, len(t))
            elif op == "fork":
                for bm in (nat, ora):
                    bm.fork(s, next_id)
                toks[next_id] = list(t)
                next_id += 1
            elif op == "trunc":
                n = int(rng.integers(0, len(t) + 1))
                for bm in (nat, ora):
                    bm.truncate(s, n)
                toks[s] = t[:n]
            else:
                for bm in (nat, ora):
                    bm.free(s)
                del toks[s]
        assert {s: nat.block_table(s) for s in toks} == {s: ora.block_table(s) for s in toks}, step
        assert [int(x) for x in nat.alloc.ref] == list(ora.alloc.ref), step
        assert list(nat.alloc.free) == list(ora.alloc.free), step
        assert list(nat.alloc.evictable) == list(ora.alloc.lru), step
        assert nat.alloc.block_hash == ora.alloc.hash_of, step
        assert {s: list(nat.tables[s].hashes) for s in toks} == {s: ora.hashes[s] for s in toks}, step
