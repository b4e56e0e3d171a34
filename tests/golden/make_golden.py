"""Generate the golden fixtures in this folder by running pagellm itself.

Run with ``PAGELLM_SRC`` naming the ``src`` directory of a pagellm checkout:

    PAGELLM_SRC=<pagellm checkout>/src python tests/golden/make_golden.py          # all
    PAGELLM_SRC=<pagellm checkout>/src python tests/golden/make_golden.py engine   # engine_*.npz only

Every fixture records seeded inputs together with the outputs of pagellm's own
functions on them (``pagellm.cache.paged``, ``pagellm.model.transformer``). The tests
replay them against the CPU oracle (``oracle/paged_oracle.py``) and, on a GPU, against
the CUDA path. Nothing at test time imports pagellm: the fixtures are the pin.
"""

from __future__ import annotations

import json
import os
import random
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
if not os.environ.get("PAGELLM_SRC"):
    sys.exit("set PAGELLM_SRC to the src directory of a pagellm checkout")
sys.path.insert(0, os.environ["PAGELLM_SRC"])

from pagellm.cache.paged import (  # noqa: E402
    BlockManager,
    OutOfBlocks,
    PagedBatch,
    PagedKVPool,
    batched_decode_attention,
    paged_attention,
    slot_mapping,
)
from pagellm.model.transformer import ModelConfig, causal_attention  # noqa: E402


def bf16_round(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return r.view(np.float32)


def paged_attention_cases():
    """Shapes of pagellm's ``tests/unit/test_paged.py:18-32`` plus extra windows."""
    out = {}
    rng = np.random.default_rng(1234)
    cases = [(1, 1, 4), (37, 1, 8), (37, 37, 8), (64, 5, 16), (9, 3, 4), (100, 17, 16), (16, 1, 16)]
    for ci, (ctx, n, bs) in enumerate(cases):
        H, KVH, d = 4, 2, 8
        nblk = -(-ctx // bs)
        table = rng.permutation(nblk + 5)[:nblk]
        kp = rng.standard_normal((nblk + 5, bs, KVH, d))
        vp = rng.standard_normal((nblk + 5, bs, KVH, d))
        q = rng.standard_normal((n, H, d))
        k = np.concatenate([kp[b] for b in table])[:ctx]
        v = np.concatenate([vp[b] for b in table])[:ctx]
        out[f"c{ci}_meta"] = np.array([ctx, n, bs], np.int64)
        out[f"c{ci}_table"] = table.astype(np.int64)
        out[f"c{ci}_kp"], out[f"c{ci}_vp"], out[f"c{ci}_q"] = kp, vp, q
        out[f"c{ci}_dense"] = causal_attention(q, k, v, ctx - n)
        out[f"c{ci}_paged"] = paged_attention(q, kp, vp, table.tolist(), ctx, ctx - n)
    out["ncases"] = np.array(len(cases))
    return out


def batched_decode_case():
    """``tests/unit/test_paged.py:150-162``: garbage padding must not leak."""
    rng = np.random.default_rng(1234)
    H, KVH, d = 4, 2, 8
    lens = np.array([1, 7, 33, 20])
    lmax = int(lens.max())
    q = rng.standard_normal((len(lens), H, d))
    k = rng.standard_normal((len(lens), lmax, KVH, d))
    v = rng.standard_normal((len(lens), lmax, KVH, d))
    valid = np.arange(lmax)[None, :] < lens[:, None]
    k[~valid] = 1e3
    return dict(lens=lens, q=q, k=k, v=v, valid=valid, out=batched_decode_attention(q, k, v, valid))


def _step_case(rng, H, KVH, d, bs, num_blocks, ctx_lens, n_new, dtype, attn, batch_decode=True,
               round_bf16=False):
    """One PagedBatch step on a scattered pool; returns inputs and pagellm's outputs.

    Only the context rows each sequence reads are stored (with their slots), so the
    fixture stays small: the replay scatters them into a zero pool.
    """
    cfg = ModelConfig(vocab_size=8, dim=H * d, n_layers=1, n_heads=H, n_kv_heads=KVH)
    pool = PagedKVPool(cfg, num_blocks, bs, dtype)
    perm = rng.permutation(num_blocks)
    tables, used = [], 0
    for L in ctx_lens:
        nb = -(-int(L) // bs)
        tables.append(perm[used:used + nb].tolist())
        used += nb
    starts = [int(L) - int(n) for L, n in zip(ctx_lens, n_new)]
    # cached context (positions < start) is already in the pool
    ctx_slots = np.concatenate(
        [slot_mapping(t, np.arange(s), bs) for t, s in zip(tables, starts)] + [np.zeros(0, np.int64)]
    ).astype(np.int64)
    kc = rng.standard_normal((len(ctx_slots), KVH, d)).astype(dtype)
    vc = rng.standard_normal((len(ctx_slots), KVH, d)).astype(dtype)
    N = int(sum(n_new))
    q = rng.standard_normal((N, H, d)).astype(dtype)
    k = rng.standard_normal((N, KVH, d)).astype(dtype)
    v = rng.standard_normal((N, KVH, d)).astype(dtype)
    if round_bf16:
        kc, vc, k, v = (bf16_round(a) for a in (kc, vc, k, v))
    pool.k_flat[0, ctx_slots] = kc
    pool.v_flat[0, ctx_slots] = vc
    kv = PagedBatch(pool, tables, starts, list(map(int, n_new)), attn, batch_decode)
    out = kv.write_and_attend(0, q, k, v)
    indptr = np.concatenate([[0], np.cumsum([len(t) for t in tables])]).astype(np.int64)
    if round_bf16:  # stored as bf16 bit patterns: exact and half the size
        kc, vc, k, v = ((a.view(np.uint32) >> np.uint32(16)).astype(np.uint16) for a in (kc, vc, k, v))
    return dict(
        dims=np.array([H, KVH, d, bs, num_blocks], np.int64),
        indptr=indptr,
        ids=np.concatenate([np.asarray(t, np.int64) for t in tables]),
        starts=np.array(starts, np.int64),
        n_new=np.array(n_new, np.int64),
        ctx_slots=ctx_slots,
        kc=kc, vc=vc, q=q, k=k, v=v,
        positions=kv.positions,
        slots=kv.slots,
        out=out,
    )


def step_cases():
    res = {}
    rng = np.random.default_rng(7)
    # C1: decode fp32, B=8, H=4, KVH=2, d=32, bs=16, L ~ U{1..256}, 256-block pool
    L = rng.integers(1, 257, 8)
    res["c1_gather"] = _step_case(rng, 4, 2, 32, 16, 256, L, [1] * 8, np.float32, "gather")
    L = rng.integers(1, 257, 8)
    res["c1_paged"] = _step_case(rng, 4, 2, 32, 16, 256, L, [1] * 8, np.float32, "paged")
    # mixed step: prefill chunks, a verify window and decodes in one batch
    L = np.array([40, 3, 97, 1, 64, 130])
    n = [40, 1, 17, 1, 5, 1]
    res["mixed_gather"] = _step_case(rng, 4, 2, 32, 16, 64, L, n, np.float32, "gather")
    res["mixed_paged"] = _step_case(rng, 4, 2, 32, 16, 64, L, n, np.float32, "paged")
    # bf16-rounded K/V, Llama-3-8B attention shape, short contexts
    L = rng.integers(1, 120, 4)
    res["bf16_c2shape"] = _step_case(rng, 32, 8, 128, 16, 128, L, [1] * 4, np.float32, "gather",
                                     round_bf16=True)
    L = np.array([53, 70])
    res["bf16_verify"] = _step_case(rng, 32, 8, 128, 16, 40, L, [5, 5], np.float32, "gather",
                                    round_bf16=True)
    return res


def fork_case():
    """Forks over a shared prefix, C4's shape in small: one request's 100-token prompt is
    prefilled, forked 4 ways (BlockManager.fork), each fork's ensure_capacity copy-on-writes
    the shared partial block (PagedKVPool.copy_block), then one gather step verifies 5
    tokens per fork. bf16-rounded K/V/q-independent data, Llama-3-8B attention shape."""
    rng = np.random.default_rng(21)
    H, KVH, d, bs, nb, P, forks, nv = 32, 8, 128, 16, 48, 100, 4, 5
    cfg = ModelConfig(vocab_size=8, dim=H * d, n_layers=1, n_heads=H, n_kv_heads=KVH)
    pool = PagedKVPool(cfg, nb, bs, np.float32)
    bm = BlockManager(nb, bs)
    prompt = [int(t) for t in rng.integers(0, 8, P)]
    bm.allocate(0, prompt)
    ctx_slots = slot_mapping(bm.block_table(0), np.arange(P), bs).astype(np.int64)
    kc = bf16_round(rng.standard_normal((P, KVH, d)).astype(np.float32))
    vc = bf16_round(rng.standard_normal((P, KVH, d)).astype(np.float32))
    pool.k_flat[0, ctx_slots] = kc
    pool.v_flat[0, ctx_slots] = vc
    for f in range(1, forks):
        bm.fork(0, f)
    pairs = []
    for f in range(forks):
        for src, dst in bm.ensure_capacity(f, P + nv, write_from=P):
            pool.copy_block(src, dst)
            pairs.append((src, dst))
    tables = [bm.block_table(f) for f in range(forks)]
    N = forks * nv
    q = rng.standard_normal((N, H, d)).astype(np.float32)
    k = bf16_round(rng.standard_normal((N, KVH, d)).astype(np.float32))
    v = bf16_round(rng.standard_normal((N, KVH, d)).astype(np.float32))
    kv = PagedBatch(pool, tables, [P] * forks, [nv] * forks, "gather", True)
    out = kv.write_and_attend(0, q, k, v)
    bits = lambda a: (a.view(np.uint32) >> np.uint32(16)).astype(np.uint16)  # noqa: E731
    return dict(
        dims=np.array([H, KVH, d, bs, nb], np.int64),
        indptr=np.concatenate([[0], np.cumsum([len(t) for t in tables])]).astype(np.int64),
        ids=np.concatenate([np.asarray(t, np.int64) for t in tables]),
        starts=np.full(forks, P, np.int64),
        n_new=np.full(forks, nv, np.int64),
        ctx_slots=ctx_slots,
        cow_pairs=np.asarray(pairs, np.int64).reshape(-1, 2),
        kc=bits(kc), vc=bits(vc), q=q, k=bits(k), v=bits(v),
        positions=kv.positions,
        slots=kv.slots,
        out=out,
    )


def slot_cases():
    rng = np.random.default_rng(3)
    out = {}
    for ci, bs in enumerate((1, 4, 16, 32)):
        nb = 12
        table = rng.permutation(1000)[:nb]
        pos = rng.integers(0, nb * bs, 50)
        out[f"s{ci}_bs"] = np.array(bs)
        out[f"s{ci}_table"] = table.astype(np.int64)
        out[f"s{ci}_pos"] = pos.astype(np.int64)
        out[f"s{ci}_slots"] = slot_mapping(table.tolist(), pos, bs)
    out["ncases"] = np.array(4)
    return out


def allocator_trace(seed: int, num_blocks: int, bs: int, prefix_caching: bool, n_ops: int):
    """Random BlockManager workload; every op's result and the resulting state."""
    r = random.Random(seed)
    bm = BlockManager(num_blocks, bs, prefix_caching)
    seqs: dict[int, list[int]] = {}
    computed: dict[int, int] = {}
    next_id = 0
    shared_prefix = [r.randrange(50) for _ in range(3 * bs + 1)]
    ops = []
    for _ in range(n_ops):
        kind = r.choice(["alloc", "alloc", "grow", "grow", "grow", "fork", "free", "can"])
        rec: dict = {"op": kind}
        if kind == "alloc" or not seqs:
            rec["op"] = "alloc"
            n = r.randrange(1, 4 * bs)
            toks = (shared_prefix[: r.randrange(len(shared_prefix))] if r.random() < 0.6 else [])
            toks = toks + [r.randrange(50) for _ in range(n)]
            sid = next_id
            next_id += 1
            rec.update(seq=sid, tokens=toks)
            try:
                cached = bm.allocate(sid, toks)
                seqs[sid] = list(toks)
                computed[sid] = len(toks)  # prefill runs in one step
                bm.mark_computed(sid, toks, len(toks))
                rec["ret"] = cached
            except OutOfBlocks:
                rec["ret"] = "OutOfBlocks"
        elif kind == "grow":
            sid = r.choice(sorted(seqs))
            add = r.randrange(1, bs + 2)
            toks = seqs[sid] + [r.randrange(50) for _ in range(add)]
            rec.update(seq=sid, tokens=toks, write_from=computed[sid])
            if bm.can_append(sid, len(toks)):
                rec["ret"] = [list(p) for p in bm.ensure_capacity(sid, len(toks), computed[sid])]
                seqs[sid] = toks
                computed[sid] = len(toks)
                bm.mark_computed(sid, toks, len(toks))
            else:
                rec["ret"] = "cannot_append"
        elif kind == "fork":
            sid = r.choice(sorted(seqs))
            child = next_id
            next_id += 1
            bm.fork(sid, child)
            seqs[child] = list(seqs[sid])
            computed[child] = computed[sid]
            rec.update(seq=sid, child=child, ret=None)
        elif kind == "free":
            sid = r.choice(sorted(seqs))
            bm.free(sid)
            del seqs[sid], computed[sid]
            rec.update(seq=sid, ret=None)
        else:
            sid = r.choice(sorted(seqs))
            n = len(seqs[sid]) + r.randrange(1, 3 * bs)
            rec.update(seq=sid, num_tokens=n, ret=bool(bm.can_append(sid, n)))
        rec["tables"] = {str(s): list(bm.block_table(s)) for s in sorted(bm.tables)}
        rec["ref"] = {str(b): int(c) for b, c in enumerate(bm.alloc.ref) if c}
        rec["free"] = list(bm.alloc.free)
        rec["evictable"] = list(bm.alloc.evictable)
        rec["num_free"] = bm.alloc.num_free
        rec["hits"] = bm.alloc.prefix_hits
        rec["queries"] = bm.alloc.prefix_queries
        ops.append(rec)
    return {"num_blocks": num_blocks, "block_size": bs, "prefix_caching": prefix_caching, "ops": ops}


ENGINE_SCENARIOS = {
    # continuous batching with prefix-cache hits (requests sharing a system prompt arrive
    # after its blocks are published) and parallel sampling n=3 (fork + copy-on-write)
    "serve": dict(config=dict(num_blocks=96, block_size=8, max_num_seqs=8, max_num_batched_tokens=256),
                  requests=[(0, "You are a helpful Shakespearean assistant.\nWho art thou?", 1, 14, 0.8, 1),
                            (2, "You are a helpful Shakespearean assistant.\nWhat news?", 1, 12, 0.0, 2),
                            (3, "ROMEO:\nBut soft", 3, 16, 1.0, 5),
                            (5, "You are a helpful Shakespearean assistant.\nSpeak!", 1, 10, 0.7, 3)]),
    # a pool too small for everyone: preemption frees blocks and recomputes prefills; the
    # block-by-block ("paged") attention mode
    "preempt": dict(config=dict(num_blocks=30, block_size=4, max_model_len=96, max_num_batched_tokens=96,
                                max_num_seqs=8, attn="paged"),
                    requests=[(0, "First Citizen:\nBefore we proceed", 1, 40, 0.8, 11),
                              (0, "ROMEO:\nBut soft", 1, 40, 0.8, 12),
                              (0, "To be, or not", 1, 28, 0.8, 13),
                              (0, "KING RICHARD III:\nNow is the winter of our discontent", 1, 28, 0.8, 14),
                              (0, "A", 1, 28, 0.8, 15),
                              (0, "Speak, speak.", 1, 28, 0.8, 16)]),
    # chunked prefill: long prompts split over steps beside running decodes
    "chunked": dict(config=dict(num_blocks=64, block_size=16, max_num_seqs=4, max_num_batched_tokens=24,
                                enable_chunked_prefill=True),
                    requests=[(0, "First Citizen:\nBefore we proceed any further, hear me speak.\n"
                                  "All:\nSpeak, speak.\nFirst Citizen:\nYou are all resolved rather", 1, 8, 0.0, 1),
                              (1, "KING RICHARD III:\nNow is the winter of our discontent\nMade glorious summer", 1, 10,
                               0.9, 2),
                              (2, "abc", 1, 12, 0.0, 3)]),
    # the step structure only (no tensors) of a run with 16-token blocks: forks sharing
    # prompt blocks, prefix hits, chunked prefill and decodes, replayed on the GPU at a
    # tensor-core shape (bf16, head_dim 128) against the oracle
    "serve16": dict(config=dict(num_blocks=160, block_size=16, max_num_seqs=12, max_num_batched_tokens=96,
                                enable_chunked_prefill=True),
                    structure_only=True,
                    requests=[(0, "You are a helpful Shakespearean assistant. Answer in verse.\n" * 2 + "Who art thou?",
                               4, 20, 1.0, 7),
                              (3, "You are a helpful Shakespearean assistant. Answer in verse.\n" * 2 + "What news?",
                               1, 24, 0.8, 8),
                              (4, "ROMEO:\nBut soft, what light through yonder window breaks?", 3, 18, 0.9, 9),
                              (6, "You are a helpful Shakespearean assistant. Answer in verse.\n" * 2 + "Speak!",
                               2, 16, 0.7, 10)]),
}


def engine_trace(name: str) -> dict:
    """pagellm's own LLMEngine (bundled "target" model: 4 layers, H=4, KVH=2, d=32, fp32)
    run on a scenario, with every PagedBatch it builds and every copy-on-write copy it makes
    recorded: per step the copies applied before the batch, the block tables (CSR), starts,
    n_new, attention mode, positions, slots and, per layer, the q / k / v the model handed to
    write_and_attend and the output it returned (engine/llm_engine.py:201-255)."""
    import pagellm.engine.llm_engine as le
    from pagellm.engine import EngineConfig, LLMEngine, SamplingParams
    from pagellm.model.weights import load_pretrained

    sc = ENGINE_SCENARIOS[name]
    model, tok = load_pretrained("target")
    steps: list[dict] = []
    pending: list[tuple[int, int]] = []

    class RecordingBatch(PagedBatch):
        def __init__(self, pool, block_tables, starts, n_new, attn="gather", batch_decode=True):
            super().__init__(pool, block_tables, starts, n_new, attn, batch_decode)
            self._rec = {"copies": list(pending), "tables": [list(map(int, t)) for t in block_tables],
                         "starts": list(map(int, starts)), "n_new": list(map(int, n_new)), "attn": attn,
                         "batch_decode": bool(batch_decode), "positions": self.positions.copy(),
                         "slots": self.slots.copy(), "layers": []}
            pending.clear()
            steps.append(self._rec)

        def write_and_attend(self, layer, q, k, v):
            out = super().write_and_attend(layer, q, k, v)
            self._rec["layers"].append((layer, q.copy(), k.copy(), v.copy(), out.copy()))
            return out

    saved = le.PagedBatch
    le.PagedBatch = RecordingBatch
    try:
        eng = LLMEngine(model, tok, EngineConfig(**sc["config"]))
        copy_block = eng.pool.copy_block

        def recording_copy(src, dst):
            pending.append((int(src), int(dst)))
            copy_block(src, dst)

        eng.pool.copy_block = recording_copy
        todo = sorted(sc["requests"], key=lambda r: r[0])
        step_no = 0
        while todo or eng.has_unfinished():
            while todo and todo[0][0] <= step_no:
                _, prompt, n, max_tokens, temp, seed = todo.pop(0)
                eng.add_request(prompt, SamplingParams(n=n, max_tokens=max_tokens, temperature=temp, seed=seed))
            eng.step()
            step_no += 1
            assert step_no < 2000
        stats = {"preemptions": eng.scheduler.num_preemptions, "cow_copies": eng.stats.cow_copies,
                 "prefix_hits": eng.bm.alloc.prefix_hits, "cached_prompt_tokens": eng.stats.cached_prompt_tokens,
                 "steps": eng.stats.steps}
    finally:
        le.PagedBatch = saved
    cfg = model.cfg
    out = {"dims": np.array([cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                             eng.config.num_blocks, eng.config.block_size], np.int64),
           "nsteps": np.array(len(steps)), "stats": np.array(json.dumps(stats))}
    for i, st in enumerate(steps):
        lens = np.array([len(t) for t in st["tables"]], np.int64)
        ip = np.zeros(len(lens) + 1, np.int64)
        np.cumsum(lens, out=ip[1:])
        out[f"s{i}_copies"] = np.array(st["copies"], np.int64).reshape(-1, 2)
        out[f"s{i}_indptr"] = ip
        out[f"s{i}_ids"] = np.array([b for t in st["tables"] for b in t], np.int64)
        out[f"s{i}_starts"] = np.array(st["starts"], np.int64)
        out[f"s{i}_n_new"] = np.array(st["n_new"], np.int64)
        out[f"s{i}_mode"] = np.array([st["attn"] == "paged", st["batch_decode"]], np.int64)
        out[f"s{i}_positions"] = st["positions"]
        out[f"s{i}_slots"] = st["slots"]
        assert [l_[0] for l_ in st["layers"]] == list(range(cfg.n_layers))
        if sc.get("structure_only"):
            continue
        for key, j in (("q", 1), ("k", 2), ("v", 3), ("out", 4)):
            out[f"s{i}_{key}"] = np.stack([l_[j] for l_ in st["layers"]]).astype(np.float32)
    return out


def main(only=None):
    if only == "engine":
        for name in ENGINE_SCENARIOS:
            np.savez_compressed(HERE / f"engine_{name}.npz", **engine_trace(name))
        print("wrote", sorted(p.name for p in HERE.iterdir() if p.name.startswith("engine_")))
        return
    for name in ENGINE_SCENARIOS:
        np.savez_compressed(HERE / f"engine_{name}.npz", **engine_trace(name))
    np.savez_compressed(HERE / "paged_attention_cases.npz", **paged_attention_cases())
    np.savez_compressed(HERE / "batched_decode.npz", **batched_decode_case())
    for name, case in step_cases().items():
        np.savez_compressed(HERE / f"step_{name}.npz", **case)
    np.savez_compressed(HERE / "step_bf16_forks.npz", **fork_case())
    np.savez_compressed(HERE / "slot_mapping.npz", **slot_cases())
    traces = [
        allocator_trace(11, 24, 4, True, 300),
        allocator_trace(12, 24, 4, False, 300),
        allocator_trace(13, 48, 16, True, 200),
    ]
    (HERE / "allocator_traces.json").write_text(json.dumps(traces, separators=(",", ":")))
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".npz", ".json")))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else None)
