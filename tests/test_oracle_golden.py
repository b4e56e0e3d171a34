"""Pin the CPU oracle to pagellm's own outputs (golden fixtures made by running pagellm).

These run without a GPU. Tolerances: float64 cases 1e-12 absolute (pagellm's own
``tests/unit/test_paged.py:32``); float32 steps 1e-5 relative / 1e-6 absolute; integer
index work bit-exact.
"""

from __future__ import annotations

import numpy as np
import pytest
from conftest import load_npz, load_traces, step_inputs

from oracle import paged_oracle as po

STEP_CASES = ["c1_gather", "c1_paged", "mixed_gather", "mixed_paged", "bf16_c2shape", "bf16_verify"]


def test_paged_attention_cases_dense_and_online():
    z = load_npz("paged_attention_cases.npz")
    for ci in range(int(z["ncases"])):
        ctx, n, bs = (int(x) for x in z[f"c{ci}_meta"])
        table = z[f"c{ci}_table"].tolist()
        kp, vp, q = z[f"c{ci}_kp"], z[f"c{ci}_vp"], z[f"c{ci}_q"]
        k = np.concatenate([kp[b] for b in table])[:ctx]
        v = np.concatenate([vp[b] for b in table])[:ctx]
        dense = po.attention_dense(q, k, v, ctx - n)
        online = po.attention_online_blocks(q, kp, vp, table, ctx, ctx - n)
        np.testing.assert_allclose(dense, z[f"c{ci}_dense"], atol=1e-12, rtol=0)
        np.testing.assert_allclose(online, z[f"c{ci}_paged"], atol=1e-12, rtol=0)


def test_padded_decode_ignores_garbage():
    z = load_npz("batched_decode.npz")
    got = po.attention_padded_decode(z["q"], z["k"], z["v"], z["valid"])
    np.testing.assert_allclose(got, z["out"], atol=1e-12, rtol=0)


def test_slot_mapping_bit_exact():
    z = load_npz("slot_mapping.npz")
    for ci in range(int(z["ncases"])):
        got = po.slot_mapping(z[f"s{ci}_table"], z[f"s{ci}_pos"], int(z[f"s{ci}_bs"]))
        assert got.dtype == np.int64
        np.testing.assert_array_equal(got, z[f"s{ci}_slots"])


@pytest.mark.parametrize("name", STEP_CASES)
def test_write_and_attend_step(name):
    c = step_inputs(load_npz(f"step_{name}.npz"))
    attn = "paged" if name.endswith("paged") else "gather"
    meta = po.StepMeta(c["tables"], c["starts"], c["n_new"], c["bs"], attn=attn)
    np.testing.assert_array_equal(meta.positions, c["positions"])
    np.testing.assert_array_equal(meta.slots, c["slots"])
    kpool = np.zeros((c["num_blocks"], c["bs"], c["KVH"], c["d"]), np.float32)
    vpool = np.zeros_like(kpool)
    kf = kpool.reshape(-1, c["KVH"], c["d"])
    vf = vpool.reshape(-1, c["KVH"], c["d"])
    kf[c["ctx_slots"]] = c["kc"]
    vf[c["ctx_slots"]] = c["vc"]
    out = po.write_and_attend(kf, vf, meta, c["q"], c["k"], c["v"], kpool, vpool)
    np.testing.assert_allclose(out, c["out"], rtol=1e-5, atol=1e-6)
    # the appended rows are in the pool, bit for bit
    np.testing.assert_array_equal(kf[c["slots"]], c["k"])
    np.testing.assert_array_equal(vf[c["slots"]], c["v"])


def test_fork_cow_verify_step():
    """pagellm's fork + copy-on-write + verify step (step_bf16_forks.npz): the recorded CoW
    pairs replayed with the oracle's copy_blocks, then the step."""
    z = load_npz("step_bf16_forks.npz")
    c = step_inputs(z)
    meta = po.StepMeta(c["tables"], c["starts"], c["n_new"], c["bs"], attn="gather")
    np.testing.assert_array_equal(meta.positions, c["positions"])
    np.testing.assert_array_equal(meta.slots, c["slots"])
    kpool = np.zeros((c["num_blocks"], c["bs"], c["KVH"], c["d"]), np.float32)
    vpool = np.zeros_like(kpool)
    kf = kpool.reshape(-1, c["KVH"], c["d"])
    vf = vpool.reshape(-1, c["KVH"], c["d"])
    kf[c["ctx_slots"]] = c["kc"]
    vf[c["ctx_slots"]] = c["vc"]
    pairs = [tuple(map(int, p)) for p in z["cow_pairs"]]
    assert len(pairs) == 3  # 4 forks: the first 3 writers copy, the last keeps the block
    po.copy_blocks(kpool[None], vpool[None], pairs)
    out = po.write_and_attend(kf, vf, meta, c["q"], c["k"], c["v"], kpool, vpool)
    np.testing.assert_allclose(out, c["out"], rtol=1e-5, atol=1e-6)


def test_bf16_round_is_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e-3, 65504.0, 1.0 + 2 ** -8], np.float32)
    bits = po.bf16_bits(x)
    # 1 + 2^-8 is a tie between 1.0 and 1.0078125: even mantissa (1.0) wins
    assert bits[-1] == 0x3F80
    back = po.bf16_round(x)
    assert np.all(np.abs(back - x) <= np.abs(x) * 2.0 ** -8)
    # round trip of exactly representable values is the identity
    y = po.bf16_round(np.random.default_rng(0).standard_normal(1000).astype(np.float32))
    np.testing.assert_array_equal(po.bf16_round(y), y)


def _replay(trace, manager_cls, out_of_blocks):
    bm = manager_cls(trace["num_blocks"], trace["block_size"], trace["prefix_caching"])
    for step, rec in enumerate(trace["ops"]):
        op = rec["op"]
        if op == "alloc":
            try:
                got = bm.allocate(rec["seq"], rec["tokens"])
                bm.mark_computed(rec["seq"], rec["tokens"], len(rec["tokens"]))
            except out_of_blocks:
                got = "OutOfBlocks"
        elif op == "grow":
            toks = rec["tokens"]
            if bm.can_append(rec["seq"], len(toks)):
                got = [list(p) for p in bm.ensure_capacity(rec["seq"], len(toks), rec["write_from"])]
                bm.mark_computed(rec["seq"], toks, len(toks))
            else:
                got = "cannot_append"
        elif op == "fork":
            bm.fork(rec["seq"], rec["child"])
            got = None
        elif op == "free":
            bm.free(rec["seq"])
            got = None
        else:
            got = bool(bm.can_append(rec["seq"], rec["num_tokens"]))
        assert got == rec["ret"], (step, op)
        tables = {str(s): list(bm.block_table(s)) for s in sorted(_seq_ids(bm))}
        assert tables == rec["tables"], step
        ref = {str(b): int(c) for b, c in enumerate(_refs(bm)) if c}
        assert ref == rec["ref"], step
        assert list(_free_list(bm)) == rec["free"], step
        assert list(_evictable(bm)) == rec["evictable"], step
        assert bm.alloc.num_free == rec["num_free"], step
        assert (bm.alloc.prefix_hits, bm.alloc.prefix_queries) == (rec["hits"], rec["queries"])


def _seq_ids(bm):
    return bm.blocks.keys() if hasattr(bm, "blocks") else bm.tables.keys()


def _refs(bm):
    return bm.alloc.ref


def _free_list(bm):
    return bm.alloc.free


def _evictable(bm):
    return bm.alloc.lru if hasattr(bm.alloc, "lru") else bm.alloc.evictable


@pytest.mark.parametrize("ti", [0, 1, 2])
def test_oracle_block_manager_replays_pagellm(ti):
    _replay(load_traces()[ti], po.OracleBlockManager, po.OracleOutOfBlocks)


@pytest.mark.parametrize("name", ["serve", "preempt", "chunked"])
def test_oracle_replays_pagellm_engine(name):
    """pagellm's own LLMEngine runs (tests/golden/engine_*.npz: 4 layers, prefix hits, an n=3
    fork with copy-on-write, preemption with recompute, chunked prefill) replayed through the
    oracle on a zero-filled multi-layer pool: every step's positions and slots bit-exact,
    every layer's output within 1e-5 of its scale of pagellm's (float32 on both sides)."""
    from engine_trace import OraclePool, Trace, assert_close_scaled

    tr = Trace(name)
    pool = OraclePool(tr.layers, tr.num_blocks, tr.bs, tr.KVH, tr.d)
    for st in tr.steps:
        meta = po.StepMeta(st.tables, st.starts, st.n_new, tr.bs, st.batch_decode, st.attn)
        np.testing.assert_array_equal(meta.positions, st.positions)
        np.testing.assert_array_equal(meta.slots, st.slots)
        inputs = [(st.q[li], st.k[li], st.v[li]) for li in range(tr.layers)]
        for li, out in pool.step(st, inputs):
            assert_close_scaled(out, st.out[li])


def test_engine_traces_cover_the_engine_paths():
    """What the recorded runs exercise (so a regenerated fixture cannot silently lose it)."""
    from engine_trace import Trace

    serve, pre, chunk, s16 = (Trace(n) for n in ("serve", "preempt", "chunked", "serve16"))
    assert serve.stats["cow_copies"] >= 2 and serve.stats["prefix_hits"] > 0
    assert pre.stats["preemptions"] > 0 and any(s.attn == "paged" for s in pre.steps)
    assert max(max(s.n_new) for s in chunk.steps) <= 24 < sum(s.rows for s in chunk.steps)
    assert any(len(s.copies) for s in s16.steps) and max(max(s.n_new) for s in s16.steps) >= 16
    assert all(t.layers == 4 and (t.H, t.KVH, t.d) == (4, 2, 32) for t in (serve, pre, chunk))
