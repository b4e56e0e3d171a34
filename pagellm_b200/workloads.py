"""Seeded synthetic workloads for the paged KV-cache hot path.

Five configurations, C1..C5, with the shapes the pagellm KV-cache path is benchmarked on
(single layer; block tables drawn from a random permutation of the pool, so blocks are
scattered):

* C1 - CPU-sized decode check: B=8, H=4, KVH=2, d=32, fp32, L ~ U{1..256}, 256-block pool.
* C2 - Llama-3-8B decode: B=64, H=32, KVH=8, d=128, bf16, L ~ U{512..4096},
  pool = ceil(1.25 * total blocks).
* C3 - mixed chunked-prefill step: 16 decode rows (L ~ U{256..2048}) plus one 512-query
  chunk at positions 1024..1535 of a sequence whose first 1024 tokens are cached.
* C4 - prefix sharing + copy-on-write + speculative verify: 64 requests share a 2048-token
  prefix (128 shared full blocks); request j has 2048 + U{1..15} prompt tokens and is forked
  4 ways; three of the four forks copy the shared partial last block (192 copies); every
  fork then verifies 5 query tokens at positions P_j .. P_j+4.
* C5 - 70B long context: B=128, H=64, KVH=8, d=128, bf16,
  L = clip(round(lognormal(ln 8192, 0.75)), 1024, 32768) (sigma fixed here at 0.75).

``L_i`` counts the token being decoded: a decode row sits at position ``L_i - 1`` and
its K/V is appended there before attention (pagellm engine/llm_engine.py:210-226).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

C5_SIGMA = 0.75


@dataclass
class Workload:
    name: str
    H: int
    KVH: int
    D: int
    bs: int
    dtype: str  # "f32" | "bf16"
    num_blocks: int
    tables: list  # per sequence: np.ndarray[int32] of block ids
    starts: np.ndarray  # int64 [nseq]: position of the first new row
    n_new: np.ndarray  # int64 [nseq]: new rows (1 = decode)
    cow_pairs: list = field(default_factory=list)  # (src, dst) copies before the step
    notes: dict = field(default_factory=dict)

    @property
    def nseq(self) -> int:
        return len(self.tables)

    @property
    def rows(self) -> int:
        return int(self.n_new.sum())

    @property
    def ctx_lens(self) -> np.ndarray:
        return self.starts + self.n_new

    @property
    def elem_bytes(self) -> int:
        return 4 if self.dtype == "f32" else 2

    def csr(self) -> tuple[np.ndarray, np.ndarray]:
        lens = np.array([len(t) for t in self.tables], dtype=np.int64)
        indptr = np.zeros(len(lens) + 1, dtype=np.int64)
        np.cumsum(lens, out=indptr[1:])
        ids = np.concatenate(self.tables).astype(np.int32) if self.tables else np.zeros(0, np.int32)
        return indptr, ids

    def kv_read_bytes(self) -> int:
        """Algorithmic K+V bytes one step's attention reads: every row's sequence context
        once per sequence (decode) - sum_i 2 * L_i * KVH * D * elem."""
        return int(2 * self.ctx_lens.sum() * self.KVH * self.D * self.elem_bytes)

    def unique_kv_bytes(self) -> int:
        """K+V bytes of the distinct blocks the step's attention touches (shared prefix
        blocks once): what must come from HBM at least once."""
        used = set()
        for t, L in zip(self.tables, self.ctx_lens):
            used.update(np.asarray(t[: -(-int(L) // self.bs)]).tolist())
        return int(2 * len(used) * self.bs * self.KVH * self.D * self.elem_bytes)

    def attention_flops(self) -> int:
        """2 * (QK^T + PV) multiply-adds: 4 * visible keys * H * D per query row."""
        keys = 0
        for s, n in zip(self.starts, self.n_new):
            s, n = int(s), int(n)
            keys += n * s + n * (n + 1) // 2
        return int(4 * keys * self.H * self.D)

    def cow_bytes(self) -> int:
        """Bytes a copy-on-write step moves: every pair reads and writes one K and one V block."""
        return int(len(self.cow_pairs) * 2 * 2 * self.bs * self.KVH * self.D * self.elem_bytes)

    def algorithmic_bytes(self) -> int:
        """Bytes a perfect decode step moves: K/V context reads, q in + out (fp32), the
        block-table entries, the append (fp32 rows read, pool rows written) and slots."""
        e = self.elem_bytes
        ctx = self.ctx_lens
        kv = 2 * int(ctx.sum()) * self.KVH * self.D * e
        qo = self.rows * self.H * self.D * 8
        tables = int(sum(-(-int(L) // self.bs) for L in ctx)) * 4
        append = self.rows * self.KVH * self.D * 2 * (4 + e) + self.rows * 8
        return kv + qo + tables + append


def _scatter_tables(rng, ctx_lens, bs, num_blocks):
    perm = rng.permutation(num_blocks).astype(np.int32)
    tables, used = [], 0
    for L in ctx_lens:
        nb = -(-int(L) // bs)
        tables.append(perm[used:used + nb])
        used += nb
    return tables


def c1(seed: int = 0) -> Workload:
    rng = np.random.default_rng(seed)
    L = rng.integers(1, 257, 8)
    tables = _scatter_tables(rng, L, 16, 256)
    return Workload("c1", 4, 2, 32, 16, "f32", 256, tables, (L - 1).astype(np.int64),
                    np.ones(8, np.int64), notes={"L": "U{1..256}"})


def c2(seed: int = 0, batch: int = 64) -> Workload:
    rng = np.random.default_rng(seed)
    L = rng.integers(512, 4097, batch)
    need = int(sum(-(-int(x) // 16) for x in L))
    nb = math.ceil(1.25 * need)
    tables = _scatter_tables(rng, L, 16, nb)
    return Workload("c2", 32, 8, 128, 16, "bf16", nb, tables, (L - 1).astype(np.int64),
                    np.ones(batch, np.int64), notes={"L": "U{512..4096}", "pool": "1.25x"})


def c3(seed: int = 0) -> Workload:
    rng = np.random.default_rng(seed)
    Ld = rng.integers(256, 2049, 16)
    ctx = np.concatenate([Ld, [1024 + 512]])
    need = int(sum(-(-int(x) // 16) for x in ctx))
    nb = math.ceil(1.25 * need)
    tables = _scatter_tables(rng, ctx, 16, nb)
    starts = np.concatenate([Ld - 1, [1024]]).astype(np.int64)
    n_new = np.concatenate([np.ones(16, np.int64), [512]]).astype(np.int64)
    return Workload("c3", 32, 8, 128, 16, "bf16", nb, tables, starts, n_new,
                    notes={"L_decode": "U{256..2048}", "chunk": "512 queries at 1024..1535"})


def c4(seed: int = 0, requests: int = 64, forks: int = 4, verify: int = 5) -> Workload:
    """Tables as pagellm's BlockManager leaves them after prefix hits, fork and
    copy-on-write (cache/paged.py:157-263): the 128 shared prefix blocks are common to every
    fork; within a request the first forks - 1 writers get a private copy of the partial
    block, the last writer keeps the original; a block is appended when the verify window
    crosses a block boundary."""
    rng = np.random.default_rng(seed)
    bs = 16
    prefix_blocks = 2048 // bs
    extra = rng.integers(1, 16, requests)  # P_j = 2048 + extra_j
    per_fork_new = [(-(-(2048 + int(e) + verify) // bs)) - prefix_blocks - 1 for e in extra]
    need = prefix_blocks + requests * (1 + (forks - 1)) + requests * forks * max(per_fork_new + [0])
    nb = math.ceil(1.25 * need)
    perm = iter(rng.permutation(nb).astype(np.int32).tolist())
    shared = np.array([next(perm) for _ in range(prefix_blocks)], np.int32)
    tables, starts, pairs = [], [], []
    for j in range(requests):
        partial = next(perm)
        for f in range(forks):
            if f < forks - 1:
                dst = next(perm)
                pairs.append((partial, dst))
                last = dst
            else:
                last = partial
            tail = [next(perm) for _ in range(per_fork_new[j])]
            tables.append(np.concatenate([shared, [last], tail]).astype(np.int32))
            starts.append(2048 + int(extra[j]))
    n_new = np.full(len(tables), verify, np.int64)
    return Workload("c4", 32, 8, 128, bs, "bf16", nb, tables, np.array(starts, np.int64), n_new,
                    cow_pairs=pairs,
                    notes={"P": "2048+U{1..15}", "forks": forks, "verify": verify,
                           "shared_blocks": prefix_blocks})


def c5_lengths(seed: int = 0, batch: int = 128) -> np.ndarray:
    rng = np.random.default_rng(seed)
    L = np.round(rng.lognormal(math.log(8192), C5_SIGMA, batch))
    return np.clip(L, 1024, 32768).astype(np.int64)


def c5(seed: int = 0, batch: int = 128, lengths: np.ndarray | None = None,
       kv_heads: int | None = None) -> Workload:
    """Whole-batch C5 (one GPU), or a shard: ``lengths`` = this rank's sequences,
    ``kv_heads`` = this rank's KV heads in the head-sharded variant."""
    L = c5_lengths(seed, batch) if lengths is None else np.asarray(lengths, np.int64)
    kvh = 8 if kv_heads is None else kv_heads
    rng = np.random.default_rng(seed + 1)
    need = int(sum(-(-int(x) // 16) for x in L))
    nb = math.ceil(1.25 * need)
    tables = _scatter_tables(rng, L, 16, nb)
    return Workload("c5", 8 * kvh, kvh, 128, 16, "bf16", nb, tables, (L - 1).astype(np.int64),
                    np.ones(len(L), np.int64),
                    notes={"L": f"clip(lognormal(ln 8192, {C5_SIGMA}), 1024, 32768)"})


BUILDERS = {"c1": c1, "c2": c2, "c3": c3, "c4": c4, "c5": c5}


def make(name: str, seed: int = 0, **kw) -> Workload:
    return BUILDERS[name](seed=seed, **kw)
