"""Block bookkeeping with pagellm's API (src/pagellm/cache/paged.py:38-274), state in C++.

``BlockAllocator`` and ``BlockManager`` keep pagellm's names, arguments, return values and
exceptions; the free list, ref counts, evictable LRU, hash map and tables live in libpagekv
(``pk_bm_*``). Prefix hashing - the SHA-256 chain of ``block_hash``, the lookup loop of
``plan_prefix`` and the hash loop of ``mark_computed`` - stays here in Python.
"""

from __future__ import annotations

import ctypes as C
import hashlib
from collections import OrderedDict
from collections.abc import Mapping
from dataclasses import dataclass, field

import numpy as np

from .. import _lib

_PI64 = C.POINTER(C.c_int64)
_PI32 = C.POINTER(C.c_int32)
_P = C.c_void_p



class OutOfBlocks(RuntimeError):
    """The pool has no free or evictable block (paged.py:38-39)."""


def _L():
    return _lib.load()


def _ck(status: int) -> None:
    if status == 0:
        return
    msg = _L().pk_bm_last_error().decode(errors="replace")
    if status == _lib.PK_ERR_OUT_OF_BLOCKS:
        raise OutOfBlocks(msg)
    if status == _lib.PK_ERR_DOUBLE_FREE:
        raise RuntimeError(msg)
    if status == _lib.PK_ERR_NOT_FOUND:
        raise KeyError(msg)
    if status == _lib.PK_ERR_OUT_OF_RANGE:
        raise IndexError(msg)
    raise ValueError(msg)


def block_hash(parent: bytes, tokens) -> bytes:
    """Digest of a full block chained onto everything before it (paged.py:120-131):
    SHA-256 over the parent digest followed by the tokens as little-endian int64."""
    h = hashlib.sha256(parent)
    h.update(np.asarray(tokens, dtype=np.int64).tobytes())
    return h.digest()


class _Native:
    """Owns one pk_block_manager."""

    def __init__(self, num_blocks: int, block_size: int, enable_prefix_caching: bool):
        h = _P()
        _ck(_L().pk_bm_create(int(num_blocks), int(block_size), int(bool(enable_prefix_caching)),
                              C.byref(h)))
        self.ptr = h.value
        r = _PI64()
        _ck(_L().pk_bm_refcounts(self.ptr, C.byref(r)))
        self.ref = np.ctypeslib.as_array(r, shape=(int(num_blocks),)) if num_blocks else np.zeros(0, np.int64)

    def counts(self) -> list[int]:
        c = (C.c_int64 * 7)()
        _ck(_L().pk_bm_counts(self.ptr, c))
        return list(c)

    def __del__(self):
        try:
            if self.ptr:
                _L().pk_bm_destroy(self.ptr)
                self.ptr = 0
        except Exception:
            pass


def _ids_list(fn, ptr, *args) -> list[int]:
    n = C.c_int64()
    _ck(fn(ptr, *args, None, 0, C.byref(n)))
    buf = (C.c_int32 * max(1, n.value))()
    _ck(fn(ptr, *args, buf, n.value, C.byref(n)))
    return list(buf[: n.value])


class BlockAllocator:
    """Free list, ref counts and prefix-hash cache (paged.py:47-117)."""

    def __init__(self, num_blocks: int, enable_prefix_caching: bool = True, *, _native=None):
        self.num_blocks = int(num_blocks)
        self.enable_prefix_caching = bool(enable_prefix_caching)
        self._n = _native if _native is not None else _Native(num_blocks, 1, enable_prefix_caching)

    # -- state views (live or freshly copied) ------------------------------
    @property
    def ref(self) -> np.ndarray:
        """Live int64 view of the native ref counts."""
        return self._n.ref

    @property
    def free(self) -> list[int]:
        return _ids_list(_L().pk_bm_free_list, self._n.ptr)

    @property
    def evictable(self) -> OrderedDict:
        return OrderedDict((b, None) for b in _ids_list(_L().pk_bm_evictable_list, self._n.ptr))

    def _hash_of(self, b: int) -> bytes | None:
        n = C.c_int64()
        _ck(_L().pk_bm_block_hash(self._n.ptr, int(b), None, 0, C.byref(n)))
        if n.value < 0:
            return None
        buf = C.create_string_buffer(max(1, n.value))
        _ck(_L().pk_bm_block_hash(self._n.ptr, int(b), buf, n.value, C.byref(n)))
        return buf.raw[: n.value]

    @property
    def block_hash(self) -> dict:
        out = {}
        for b in range(self.num_blocks):
            h = self._hash_of(b)
            if h is not None:
                out[b] = h
        return out

    @property
    def cached(self) -> dict:
        return {h: b for b, h in self.block_hash.items()}

    @property
    def prefix_hits(self) -> int:
        return self._n.counts()[4]

    @prefix_hits.setter
    def prefix_hits(self, v: int) -> None:
        _ck(_L().pk_bm_add_prefix_stats(self._n.ptr, int(v) - self.prefix_hits, 0))

    @property
    def prefix_queries(self) -> int:
        return self._n.counts()[5]

    @prefix_queries.setter
    def prefix_queries(self, v: int) -> None:
        _ck(_L().pk_bm_add_prefix_stats(self._n.ptr, 0, int(v) - self.prefix_queries))

    # -- capacity ----------------------------------------------------------
    @property
    def num_free(self) -> int:
        return self._n.counts()[0]

    @property
    def num_used(self) -> int:
        return self.num_blocks - self.num_free

    # -- alloc / free ------------------------------------------------------
    def allocate(self) -> int:
        b = C.c_int32()
        _ck(_L().pk_bm_allocate_block(self._n.ptr, C.byref(b)))
        return b.value

    def incref(self, b: int) -> None:
        _ck(_L().pk_bm_incref(self._n.ptr, int(b)))

    def decref(self, b: int) -> None:
        _ck(_L().pk_bm_decref(self._n.ptr, int(b)))

    # -- prefix cache ------------------------------------------------------
    def lookup(self, h: bytes) -> int | None:
        b = C.c_int32()
        _ck(_L().pk_bm_lookup(self._n.ptr, h, len(h), C.byref(b)))
        return None if b.value < 0 else b.value

    def register(self, b: int, h: bytes) -> None:
        _ck(_L().pk_bm_register(self._n.ptr, int(b), h, len(h)))


@dataclass
class BlockTable:
    """A sequence's physical blocks and the digests of its leading full blocks (paged.py:139-144)."""

    blocks: list[int] = field(default_factory=list)
    hashes: list[bytes] = field(default_factory=list)


class _TablesView(Mapping):
    """Read-only ``seq_id -> BlockTable`` view of the native tables (``BlockManager.tables``)."""

    def __init__(self, bm: "BlockManager"):
        self._bm = bm

    def _ids(self) -> list[int]:
        n = C.c_int64()
        _ck(_L().pk_bm_seq_ids(self._bm._n.ptr, None, 0, C.byref(n)))
        buf = (C.c_int64 * max(1, n.value))()
        _ck(_L().pk_bm_seq_ids(self._bm._n.ptr, buf, n.value, C.byref(n)))
        return list(buf[: n.value])

    def __getitem__(self, seq_id):
        return BlockTable(self._bm.block_table(seq_id), self._bm._chain(seq_id))

    def __contains__(self, seq_id) -> bool:
        n = C.c_int64()
        return _L().pk_bm_table(self._bm._n.ptr, int(seq_id), None, 0, C.byref(n)) == 0

    def __iter__(self):
        return iter(self._ids())

    def __len__(self) -> int:
        return self._bm._n.counts()[6]


class BlockManager:
    """Per-sequence block tables on top of the allocator (paged.py:147-274)."""

    def __init__(self, num_blocks: int, block_size: int, enable_prefix_caching: bool = True):
        self.block_size = int(block_size)
        self._n = _Native(num_blocks, block_size, enable_prefix_caching)
        self.alloc = BlockAllocator(num_blocks, enable_prefix_caching, _native=self._n)
        self.tables = _TablesView(self)

    @property
    def handle(self) -> int:
        return self._n.ptr

    def blocks_needed(self, num_tokens: int) -> int:
        return -(-num_tokens // self.block_size)

    # -- admission ---------------------------------------------------------
    def plan_prefix(self, tokens) -> tuple[list[int], list[bytes]]:
        """Cached blocks for the longest full-block prefix of ``tokens``, at most
        (len-1)//block_size of them: the last prompt token is always recomputed (paged.py:157-178)."""
        if not self.alloc.enable_prefix_caching:
            return [], []
        bs = self.block_size
        hits: list[int] = []
        chain: list[bytes] = []
        h = b""
        for i in range((len(tokens) - 1) // bs):
            h = block_hash(h, tokens[i * bs:(i + 1) * bs])
            b = self.alloc.lookup(h)
            if b is None:
                break
            hits.append(b)
            chain.append(h)
        return hits, chain

    def can_allocate(self, tokens) -> bool:
        hits, _ = self.plan_prefix(tokens)
        revived = sum(1 for b in hits if self.alloc.ref[b] == 0)
        return self.blocks_needed(len(tokens)) - len(hits) + revived <= self.alloc.num_free

    def allocate(self, seq_id: int, tokens) -> int:
        """Create the table of a new sequence; returns how many leading tokens are cached."""
        hits, chain = self.plan_prefix(tokens)
        arr = (C.c_int32 * max(1, len(hits)))(*hits)
        hlen = len(chain[0]) if chain else 0
        if any(len(h) != hlen for h in chain):
            raise ValueError("digests of one chain must have one length")
        cached = C.c_int64()
        _ck(_L().pk_bm_seq_allocate(self._n.ptr, int(seq_id), len(tokens), arr, len(hits),
                                    b"".join(chain), hlen, C.byref(cached)))
        return cached.value

    # -- growth ------------------------------------------------------------
    def can_append(self, seq_id: int, num_tokens: int) -> bool:
        ok = C.c_int()
        _ck(_L().pk_bm_can_append(self._n.ptr, int(seq_id), int(num_tokens), C.byref(ok)))
        return bool(ok.value)

    def ensure_capacity(self, seq_id: int, num_tokens: int, write_from: int) -> list[tuple[int, int]]:
        """Grow to ``num_tokens`` and privatise the blocks written from ``write_from`` on;
        returns the (src, dst) copies to run before the forward pass (paged.py:215-239)."""
        n = C.c_int64()
        cap = max(1, len(self.block_table(seq_id)))
        buf = (C.c_int64 * (2 * cap))()
        _ck(_L().pk_bm_ensure_capacity(self._n.ptr, int(seq_id), int(num_tokens), int(write_from),
                                       buf, cap, C.byref(n)))
        return [(buf[2 * i], buf[2 * i + 1]) for i in range(n.value)]

    def _chain(self, seq_id) -> list[bytes]:
        n, ln = C.c_int64(), C.c_int64()
        _ck(_L().pk_bm_seq_hashes(self._n.ptr, int(seq_id), C.byref(n), None, 0, C.byref(ln)))
        out = []
        for i in range(n.value):
            _ck(_L().pk_bm_seq_hash_at(self._n.ptr, int(seq_id), i, None, 0, C.byref(ln)))
            buf = C.create_string_buffer(max(1, ln.value))
            _ck(_L().pk_bm_seq_hash_at(self._n.ptr, int(seq_id), i, buf, ln.value, C.byref(ln)))
            out.append(buf.raw[: ln.value])
        return out

    def mark_computed(self, seq_id: int, tokens, num_computed: int) -> None:
        """Publish every newly full block in the prefix cache (paged.py:241-254)."""
        n, ln = C.c_int64(), C.c_int64()
        buf = C.create_string_buffer(64)
        _ck(_L().pk_bm_seq_hashes(self._n.ptr, int(seq_id), C.byref(n), buf, 64, C.byref(ln)))
        have = n.value
        full = num_computed // self.block_size
        if full <= have:
            return
        if ln.value > 64:
            buf = C.create_string_buffer(ln.value)
            _ck(_L().pk_bm_seq_hashes(self._n.ptr, int(seq_id), C.byref(n), buf, ln.value, C.byref(ln)))
        parent = buf.raw[: ln.value] if ln.value >= 0 else b""
        bs = self.block_size
        new = []
        for i in range(have, full):
            parent = block_hash(parent, tokens[i * bs:(i + 1) * bs])
            new.append(parent)
        _ck(_L().pk_bm_seq_push_hashes(self._n.ptr, int(seq_id), b"".join(new), len(new[0]), len(new)))

    # -- fork / free -------------------------------------------------------
    def fork(self, parent_id: int, child_id: int) -> None:
        _ck(_L().pk_bm_fork(self._n.ptr, int(parent_id), int(child_id)))

    def free(self, seq_id: int) -> None:
        _ck(_L().pk_bm_free_seq(self._n.ptr, int(seq_id)))

    def truncate(self, seq_id: int, num_tokens: int) -> None:
        """Roll the sequence back to its first ``num_tokens`` tokens (rejected speculative
        tokens): the paged form of pagellm's contiguous ``KVCache.truncate``
        (cache/contiguous.py:33-38). Blocks past them go back to the allocator, last first;
        the K/V left in the kept last block is overwritten by the next writes, which
        ``ensure_capacity(seq, n, write_from=num_tokens)`` makes private first as usual.
        ``ValueError`` if ``num_tokens`` is outside ``[0, blocks * block_size]``."""
        _ck(_L().pk_bm_truncate(self._n.ptr, int(seq_id), int(num_tokens)))

    def block_table(self, seq_id: int) -> list[int]:
        return _ids_list(_L().pk_bm_table, self._n.ptr, int(seq_id))

    def tables_csr(self, seq_ids) -> tuple[np.ndarray, np.ndarray]:
        """Block tables of ``seq_ids`` as (indptr int64, ids int32): the CSR form
        ``PagedBatch`` uploads, built natively."""
        seqs = np.ascontiguousarray(np.asarray(seq_ids, dtype=np.int64))
        indptr = np.zeros(len(seqs) + 1, dtype=np.int64)
        total = C.c_int64()
        sp = seqs.ctypes.data_as(_PI64)
        _ck(_L().pk_bm_tables_csr(self._n.ptr, sp, len(seqs), indptr.ctypes.data_as(_PI64), None, 0,
                                  C.byref(total)))
        ids = np.zeros(max(1, total.value), dtype=np.int32)
        _ck(_L().pk_bm_tables_csr(self._n.ptr, sp, len(seqs), indptr.ctypes.data_as(_PI64),
                                  ids.ctypes.data_as(_PI32), total.value, C.byref(total)))
        return indptr, ids[: total.value]
