"""CPU oracle for the paged KV-cache hot path of pagellm (TEST INFRASTRUCTURE ONLY).

This module restates, in numpy, the arithmetic of pagellm's ``cache/paged.py`` and the
attention it relies on (``model/transformer.py``). It is the checker the CUDA path is
compared against, and the CPU baseline ``bench.py`` times. Nothing in ``pagellm_b200``
imports it: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and ``--impl reference``) may use it.

Parity pin: every function here is checked against golden vectors produced by running
the reference itself (``tests/golden/make_golden.py`` imports pagellm and records inputs
and outputs; ``tests/test_oracle_golden.py`` replays them).

Citations are ``path:line`` inside the pagellm project (``src/pagellm/...``).

bf16 is not a pagellm dtype. For bf16 pools the oracle runs the fp32 arithmetic on K/V
rounded to bf16 (round to nearest, ties to even) and widened back to fp32, which is what
a bf16 pool stores.
"""

from __future__ import annotations

import math
from collections import OrderedDict, deque

import numpy as np

__all__ = [
    "bf16_round",
    "bf16_bits",
    "slot_mapping",
    "StepMeta",
    "append_rows",
    "copy_blocks",
    "attention_dense",
    "attention_padded_decode",
    "attention_online_blocks",
    "write_and_attend",
    "OracleAllocator",
    "OracleBlockManager",
    "OracleOutOfBlocks",
]


# ----------------------------------------------------------------------------- bf16

def bf16_bits(x: np.ndarray) -> np.ndarray:
    """uint16 bf16 encodings of float32 ``x``, round-to-nearest-even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    return ((u + np.uint32(0x7FFF) + lsb) >> np.uint32(16)).astype(np.uint16)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 values of ``x`` after a round trip through bf16 (RNE)."""
    return (bf16_bits(x).astype(np.uint32) << np.uint32(16)).view(np.float32).reshape(np.shape(x))


# ----------------------------------------------------------------------------- slots

def slot_mapping(block_table, positions, block_size: int) -> np.ndarray:
    """Physical slot of each logical position: table[p // bs] * bs + p % bs.

    Follows ``cache/paged.py:303-306``; int64 result.
    """
    table = np.asarray(block_table, dtype=np.int64)
    pos = np.asarray(positions, dtype=np.int64)
    blk, off = np.divmod(pos, block_size)
    return table[blk] * block_size + off


class StepMeta:
    """Per-step index math of ``PagedBatch.__init__`` (``cache/paged.py:397-439``).

    ``offsets`` - row offset of each sequence in the flat batch (``:410``)
    ``positions`` - absolute position of every new row (``:412-414``)
    ``slots`` - pool slot each new row is written to (``:415-420``)
    ``ctx_slots`` - per sequence, slots of positions 0..start+n-1 (``:422-424``)
    ``decode`` / ``prefill`` - the row-group split of ``:425-429``
    """

    def __init__(self, block_tables, starts, n_new, block_size: int, batch_decode: bool = True,
                 attn: str = "gather"):
        if attn not in ("gather", "paged"):
            raise ValueError(attn)
        self.block_size = block_size
        self.block_tables = [list(map(int, t)) for t in block_tables]
        self.starts = [int(s) for s in starts]
        self.n_new = [int(n) for n in n_new]
        self.attn = attn
        self.offsets = np.zeros(len(self.n_new) + 1, dtype=np.int64)
        np.cumsum(self.n_new, out=self.offsets[1:])
        pos_parts, slot_parts, self.ctx_slots = [], [], []
        for tbl, s, n in zip(self.block_tables, self.starts, self.n_new):
            pos = np.arange(s, s + n, dtype=np.int64)
            pos_parts.append(pos)
            slot_parts.append(slot_mapping(tbl, pos, block_size))
            self.ctx_slots.append(slot_mapping(tbl, np.arange(s + n, dtype=np.int64), block_size))
        self.positions = np.concatenate(pos_parts) if pos_parts else np.zeros(0, np.int64)
        self.slots = np.concatenate(slot_parts) if slot_parts else np.zeros(0, np.int64)
        dec = [i for i, n in enumerate(self.n_new) if n == 1]
        if attn == "gather" and batch_decode and len(dec) >= 2:
            self.decode = dec
            self.prefill = [i for i, n in enumerate(self.n_new) if n != 1]
        else:
            self.decode = []
            self.prefill = list(range(len(self.n_new)))


# ----------------------------------------------------------------------------- writes

def append_rows(k_flat_layer: np.ndarray, v_flat_layer: np.ndarray, slots, k, v) -> None:
    """Scatter new K/V rows into one layer of the flat pool (``cache/paged.py:443-444``).

    ``k_flat_layer``: (num_blocks*bs, KVH, d). Rows land at ``slots`` in order, so for
    a repeated slot the last row wins, as numpy fancy assignment does.
    """
    s = np.asarray(slots, dtype=np.int64)
    k_flat_layer[s] = np.asarray(k, dtype=k_flat_layer.dtype)
    v_flat_layer[s] = np.asarray(v, dtype=v_flat_layer.dtype)


def copy_blocks(k_pool: np.ndarray, v_pool: np.ndarray, pairs) -> None:
    """Copy-on-write block copies across all layers, in list order.

    ``k_pool``: (layers, num_blocks, bs, KVH, d). Follows ``PagedKVPool.copy_block``
    (``cache/paged.py:294-296``) as driven by ``engine/llm_engine.py:205-206``.
    """
    for src, dst in pairs:
        k_pool[:, dst] = k_pool[:, src]
        v_pool[:, dst] = v_pool[:, src]


# ----------------------------------------------------------------------------- attention

def _softmax_rows(s: np.ndarray) -> np.ndarray:
    top = s.max(axis=-1, keepdims=True)
    e = np.exp(s - top)
    return e / e.sum(axis=-1, keepdims=True)


def attention_dense(q: np.ndarray, k: np.ndarray, v: np.ndarray, q_start: int) -> np.ndarray:
    """Causal GQA attention for one sequence (``model/transformer.py:116-146``).

    q: (n, H, d) at positions q_start..q_start+n-1; k, v: (T, KVH, d) for positions
    0..T-1. Query i sees key j iff j <= q_start + i. Scores are scaled by 1/sqrt(d)
    after the dot product, max-subtracted softmax over keys, then weighted sum of V.
    """
    n, H, d = q.shape
    T, KVH, _ = k.shape
    g = H // KVH
    qh = q.reshape(n, KVH, g, d)
    scale = q.dtype.type(1.0 / math.sqrt(d))
    s = np.einsum("nkgd,tkd->kgnt", qh, k, optimize=True) * scale
    allowed = np.arange(T)[None, :] <= (q_start + np.arange(n))[:, None]
    s = np.where(allowed, s, -np.inf)
    p = _softmax_rows(s)
    o = np.einsum("kgnt,tkd->nkgd", p, v, optimize=True)
    return o.reshape(n, H, d).astype(q.dtype, copy=False)


def attention_padded_decode(q: np.ndarray, k_ctx: np.ndarray, v_ctx: np.ndarray,
                            valid: np.ndarray) -> np.ndarray:
    """One-query-per-sequence attention over padded contexts (``cache/paged.py:355-380``).

    q: (S, H, d); k_ctx, v_ctx: (S, Lmax, KVH, d); valid: (S, Lmax) bool.
    Padding positions are excluded by the mask whatever they hold.
    """
    S, H, d = q.shape
    KVH = k_ctx.shape[2]
    g = H // KVH
    qh = q.reshape(S, KVH, g, d)
    scale = q.dtype.type(1.0 / math.sqrt(d))
    s = np.einsum("skgd,slkd->skgl", qh, k_ctx, optimize=True) * scale
    s = np.where(valid[:, None, None, :], s, -np.inf)
    p = _softmax_rows(s)
    o = np.einsum("skgl,slkd->skgd", p, v_ctx, optimize=True)
    return o.reshape(S, H, d).astype(q.dtype, copy=False)


def attention_online_blocks(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray,
                            block_table, context_len: int, q_start: int) -> np.ndarray:
    """Block-at-a-time attention with a running max / sum (``cache/paged.py:309-352``).

    k_pool, v_pool: (num_blocks, bs, KVH, d) for one layer. This is the streaming
    structure of the CUDA decode kernel: per block, rescale the running sums when the
    max grows. Rows masked in every block so far keep a zero sum (guard at ``:343-347``).
    """
    n, H, d = q.shape
    bs, KVH = k_pool.shape[1], k_pool.shape[2]
    g = H // KVH
    dt = q.dtype
    qs = q.reshape(n, KVH, g, d) * dt.type(1.0 / math.sqrt(d))
    run_max = np.full((KVH, g, n), -np.inf, dtype=dt)
    run_sum = np.zeros((KVH, g, n), dtype=dt)
    acc = np.zeros((KVH, g, n, d), dtype=dt)
    qpos = q_start + np.arange(n)
    nblk = -(-context_len // bs)
    for b in range(nblk):
        phys = block_table[b]
        cnt = min(bs, context_len - b * bs)
        kb = k_pool[phys, :cnt]  # (cnt, KVH, d)
        vb = v_pool[phys, :cnt]
        s = np.einsum("nkgd,tkd->kgnt", qs, kb)
        kpos = b * bs + np.arange(cnt)
        s = np.where(kpos[None, :] <= qpos[:, None], s, -np.inf)
        new_max = np.maximum(run_max, s.max(axis=-1))
        base = np.where(np.isfinite(new_max), new_max, 0.0).astype(dt)
        w = np.exp(s - base[..., None])
        shrink = np.where(np.isfinite(run_max), np.exp(run_max - base), 0.0).astype(dt)
        run_sum = run_sum * shrink + w.sum(axis=-1)
        acc = acc * shrink[..., None] + np.einsum("kgnt,tkd->kgnd", w, vb)
        run_max = new_max
    out = acc / run_sum[..., None]
    return np.transpose(out, (2, 0, 1, 3)).reshape(n, H, d).astype(dt, copy=False)


def write_and_attend(k_flat_layer: np.ndarray, v_flat_layer: np.ndarray, meta: StepMeta,
                     q: np.ndarray, k: np.ndarray, v: np.ndarray,
                     k_pool_layer: np.ndarray | None = None,
                     v_pool_layer: np.ndarray | None = None) -> np.ndarray:
    """One layer of ``PagedBatch.write_and_attend`` (``cache/paged.py:441-464``).

    Appends the new rows, then attends: decode rows of the batch together through a
    padded gather (``:446-453``), every other sequence on its own (``:454-463``) either
    by gathered dense attention (``attn="gather"``) or block by block (``"paged"``, which
    needs the (num_blocks, bs, KVH, d) views ``k_pool_layer`` / ``v_pool_layer``).
    """
    append_rows(k_flat_layer, v_flat_layer, meta.slots, k, v)
    out = np.empty_like(q)
    if meta.decode:
        lens = [len(meta.ctx_slots[i]) for i in meta.decode]
        lmax = max(lens)
        idx = np.zeros((len(lens), lmax), dtype=np.int64)
        valid = np.zeros((len(lens), lmax), dtype=bool)
        for r, i in enumerate(meta.decode):
            idx[r, :lens[r]] = meta.ctx_slots[i]
            valid[r, :lens[r]] = True
        rows = meta.offsets[meta.decode]
        out[rows] = attention_padded_decode(q[rows], k_flat_layer[idx], v_flat_layer[idx], valid)
    for i in meta.prefill:
        a, b = int(meta.offsets[i]), int(meta.offsets[i + 1])
        s = meta.starts[i]
        if meta.attn == "paged":
            out[a:b] = attention_online_blocks(q[a:b], k_pool_layer, v_pool_layer,
                                               meta.block_tables[i], s + (b - a), s)
        else:
            cs = meta.ctx_slots[i]
            out[a:b] = attention_dense(q[a:b], k_flat_layer[cs], v_flat_layer[cs], s)
    return out


# ----------------------------------------------------------------------------- bookkeeping

class OracleOutOfBlocks(RuntimeError):
    """Pool exhausted (``cache/paged.py:38-39``)."""


class OracleAllocator:
    """Free list, ref counts and prefix-hash cache of ``BlockAllocator``
    (``cache/paged.py:47-117``), restated for replay checks of the native allocator.

    Free list: FIFO - pop from the front (``:75``), return to the back (``:101``).
    Evictable: ref==0 blocks that carry a hash, least-recently-freed evicted first
    (``:79``), revived by ``incref`` (``:87-91``).
    """

    def __init__(self, num_blocks: int, enable_prefix_caching: bool = True):
        self.num_blocks = num_blocks
        self.enable_prefix_caching = enable_prefix_caching
        self.free = deque(range(num_blocks))
        self.ref = [0] * num_blocks
        self.hash_of: dict[int, bytes] = {}
        self.block_of: dict[bytes, int] = {}
        self.lru: OrderedDict[int, None] = OrderedDict()
        self.prefix_hits = 0
        self.prefix_queries = 0

    @property
    def num_free(self) -> int:
        return len(self.free) + len(self.lru)

    @property
    def num_used(self) -> int:
        return self.num_blocks - self.num_free

    def allocate(self) -> int:
        if self.free:
            b = self.free.popleft()
        elif self.lru:
            b = next(iter(self.lru))
            del self.lru[b]
            del self.block_of[self.hash_of.pop(b)]
        else:
            raise OracleOutOfBlocks("KV cache is full")
        self.ref[b] = 1
        return b

    def incref(self, b: int) -> None:
        if self.ref[b] == 0:
            del self.lru[b]
        self.ref[b] += 1

    def decref(self, b: int) -> None:
        if self.ref[b] <= 0:
            raise RuntimeError(f"double free of block {b}")
        self.ref[b] -= 1
        if self.ref[b] == 0:
            if b in self.hash_of:
                self.lru[b] = None
            else:
                self.free.append(b)

    def lookup(self, h: bytes):
        return self.block_of.get(h) if self.enable_prefix_caching else None

    def register(self, b: int, h: bytes) -> None:
        if self.enable_prefix_caching and h not in self.block_of and b not in self.hash_of:
            self.block_of[h] = b
            self.hash_of[b] = h


def _chain_hash(parent: bytes, tokens) -> bytes:
    import hashlib

    m = hashlib.sha256(parent)
    m.update(np.asarray(tokens, dtype=np.int64).tobytes())
    return m.digest()


class OracleBlockManager:
    """Per-sequence block tables over ``OracleAllocator`` (``cache/paged.py:139-274``)."""

    def __init__(self, num_blocks: int, block_size: int, enable_prefix_caching: bool = True):
        self.block_size = block_size
        self.alloc = OracleAllocator(num_blocks, enable_prefix_caching)
        self.blocks: dict[int, list[int]] = {}
        self.hashes: dict[int, list[bytes]] = {}

    def blocks_needed(self, n: int) -> int:
        return (n + self.block_size - 1) // self.block_size

    def plan_prefix(self, tokens):
        """Longest run of cached full blocks, at most (len-1)//bs (``:157-178``)."""
        if not self.alloc.enable_prefix_caching:
            return [], []
        bs = self.block_size
        hits, chain, h = [], [], b""
        for i in range((len(tokens) - 1) // bs):
            h = _chain_hash(h, tokens[i * bs:(i + 1) * bs])
            b = self.alloc.lookup(h)
            if b is None:
                break
            hits.append(b)
            chain.append(h)
        return hits, chain

    def can_allocate(self, tokens) -> bool:
        hits, _ = self.plan_prefix(tokens)
        revive = sum(self.alloc.ref[b] == 0 for b in hits)
        return self.blocks_needed(len(tokens)) - len(hits) + revive <= self.alloc.num_free

    def allocate(self, seq_id: int, tokens) -> int:
        """New table; returns the count of leading tokens already cached (``:187-203``)."""
        if seq_id in self.blocks:
            raise ValueError(f"seq {seq_id} already has blocks")
        if not self.can_allocate(tokens):
            raise OracleOutOfBlocks("not enough blocks for prompt")
        hits, chain = self.plan_prefix(tokens)
        self.alloc.prefix_queries += (len(tokens) - 1) // self.block_size
        self.alloc.prefix_hits += len(hits)
        for b in hits:
            self.alloc.incref(b)
        fresh = [self.alloc.allocate() for _ in range(self.blocks_needed(len(tokens)) - len(hits))]
        self.blocks[seq_id] = hits + fresh
        self.hashes[seq_id] = chain
        return len(hits) * self.block_size

    def can_append(self, seq_id: int, num_tokens: int) -> bool:
        t = self.blocks[seq_id]
        need = self.blocks_needed(num_tokens) - len(t)
        if t and self.alloc.ref[t[-1]] > 1:
            need += 1
        return need <= self.alloc.num_free

    def ensure_capacity(self, seq_id: int, num_tokens: int, write_from: int):
        """Grow and privatise written blocks; returns CoW (src, dst) pairs (``:215-239``)."""
        t = self.blocks[seq_id]
        pairs = []
        for i in range(write_from // self.block_size, len(t)):
            old = t[i]
            if self.alloc.ref[old] > 1:
                new = self.alloc.allocate()
                self.alloc.decref(old)
                t[i] = new
                pairs.append((old, new))
                del self.hashes[seq_id][i:]
        while len(t) < self.blocks_needed(num_tokens):
            t.append(self.alloc.allocate())
        return pairs

    def mark_computed(self, seq_id: int, tokens, num_computed: int) -> None:
        """Register newly full blocks in the prefix cache (``:241-254``)."""
        chain = self.hashes[seq_id]
        bs = self.block_size
        h = chain[-1] if chain else b""
        for i in range(len(chain), num_computed // bs):
            h = _chain_hash(h, tokens[i * bs:(i + 1) * bs])
            chain.append(h)
            self.alloc.register(self.blocks[seq_id][i], h)

    def fork(self, parent_id: int, child_id: int) -> None:
        """Child shares every parent block (``:257-263``)."""
        for b in self.blocks[parent_id]:
            self.alloc.incref(b)
        self.blocks[child_id] = list(self.blocks[parent_id])
        self.hashes[child_id] = list(self.hashes[parent_id])

    def free(self, seq_id: int) -> None:
        """Release tail first (``:265-271``)."""
        t = self.blocks.pop(seq_id)
        self.hashes.pop(seq_id)
        for b in reversed(t):
            self.alloc.decref(b)

    def truncate(self, seq_id: int, num_tokens: int) -> None:
        """Paged speculative rollback, the paged form of pagellm's contiguous
        ``KVCache.truncate`` (``cache/contiguous.py:33-38``; paged rollback is a pagellm
        roadmap item, ``README.md:370``): keep the first ``num_tokens`` tokens; release the
        blocks past them last first (as ``free``, ``:265-271``); keep the hashes of the full
        blocks that remain; unpublish a kept partial last block that only this sequence
        holds, because its next writes change it in place."""
        t = self.blocks[seq_id]
        bs = self.block_size
        if not 0 <= num_tokens <= len(t) * bs:
            raise ValueError(f"cannot truncate a {len(t) * bs}-token table to {num_tokens}")
        keep, full = self.blocks_needed(num_tokens), num_tokens // bs
        while len(t) > keep:
            self.alloc.decref(t.pop())
        del self.hashes[seq_id][full:]
        if keep > full:
            b = t[full]
            if self.alloc.ref[b] == 1 and b in self.alloc.hash_of:
                del self.alloc.block_of[self.alloc.hash_of.pop(b)]

    def block_table(self, seq_id: int) -> list[int]:
        return self.blocks[seq_id]
