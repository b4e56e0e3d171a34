"""Parity of the CUDA path (libpagekv through its C ABI) with pagellm.

* golden fixtures recorded from pagellm itself (``tests/golden``) replayed on the GPU;
* every workload configuration C1..C5 against the CPU oracle on identical seeded inputs.

Tolerances (stated per the north-star contract):
* block tables, slot mapping, append and copy-on-write: bit-exact;
* float32 pools: |got - ref| <= 1e-5 * |ref| + 1e-6 (relative 1e-5);
* bfloat16 pools: max |got - ref| <= 2e-2 against the oracle run on the bf16-rounded K/V
  widened to float32.
"""

from __future__ import annotations

import numpy as np
import pytest
from conftest import load_npz, step_inputs
from gpu_util import (
    Shape,
    bf16_bits_of_tensor,
    gather_rows,
    make_pool,
    oracle_rows,
    step_inputs as dev_inputs,
    torch_cuda,
)

from oracle import paged_oracle as po

pytestmark = pytest.mark.gpu

F32_RTOL, F32_ATOL = 1e-5, 1e-6
BF16_ATOL = 2e-2


def _close(got, ref, bf16: bool):
    if bf16:
        err = float(np.max(np.abs(got - ref))) if got.size else 0.0
        assert err <= BF16_ATOL, f"max abs err {err}"
    else:
        np.testing.assert_allclose(got, ref, rtol=F32_RTOL, atol=F32_ATOL)


# ----------------------------------------------------------------------------- golden
@pytest.mark.parametrize("name", ["c1_gather", "c1_paged", "mixed_gather", "mixed_paged",
                                  "bf16_c2shape", "bf16_verify"])
def test_golden_step(name):
    torch = torch_cuda()
    from pagellm_b200.cache import PagedBatch, PagedKVPool

    c = step_inputs(load_npz(f"step_{name}.npz"))
    pool = PagedKVPool(Shape(1, c["KVH"], c["d"]), c["num_blocks"], c["bs"],
                       "bfloat16" if c["bf16"] else np.float32)
    idx = torch.as_tensor(c["ctx_slots"], device="cuda")
    pool.k_flat[0].index_copy_(0, idx, torch.as_tensor(c["kc"], device="cuda").to(pool.k.dtype))
    pool.v_flat[0].index_copy_(0, idx, torch.as_tensor(c["vc"], device="cuda").to(pool.v.dtype))
    attn = "paged" if name.endswith("paged") else "gather"
    batch = PagedBatch(pool, c["tables"], c["starts"], c["n_new"], attn)
    np.testing.assert_array_equal(batch.positions, c["positions"])
    np.testing.assert_array_equal(batch.slots, c["slots"])
    out = batch.write_and_attend(0, c["q"], c["k"], c["v"])
    assert out.dtype == c["q"].dtype and out.shape == c["q"].shape
    _close(out, c["out"], c["bf16"])
    kr, vr = gather_rows(pool, 0, c["slots"])
    np.testing.assert_array_equal(kr, c["k"])
    np.testing.assert_array_equal(vr, c["v"])


@pytest.mark.parametrize("mode", ["always", "off"])
def test_golden_fork_cow_verify(mode):
    """pagellm's own fork + copy-on-write + 5-token verify step (step_bf16_forks.npz) on the
    CUDA path: CoW copies through copy_blocks, then the step with the shared-prefix
    (cascade) pass forced on, and off."""
    torch = torch_cuda()
    from pagellm_b200.cache import PagedBatch, PagedKVPool

    z = load_npz("step_bf16_forks.npz")
    c = step_inputs(z)
    pool = PagedKVPool(Shape(1, c["KVH"], c["d"]), c["num_blocks"], c["bs"], "bfloat16")
    idx = torch.as_tensor(c["ctx_slots"], device="cuda")
    pool.k_flat[0].index_copy_(0, idx, torch.as_tensor(c["kc"], device="cuda").to(pool.k.dtype))
    pool.v_flat[0].index_copy_(0, idx, torch.as_tensor(c["vc"], device="cuda").to(pool.v.dtype))
    pool.copy_blocks([tuple(map(int, p)) for p in z["cow_pairs"]])
    batch = PagedBatch(pool, c["tables"], c["starts"], c["n_new"], "gather")
    batch.prefix_sharing = mode
    np.testing.assert_array_equal(batch.slots, c["slots"])
    out = batch.write_and_attend(0, c["q"], c["k"], c["v"])
    batch.check()
    assert batch.prefix_stats()["groups"] == (1 if mode == "always" else 0)
    # the shared-prefix pass reads the split-KV rows back from the output, so its result
    # comes back by a copy after the kernels; without it the kernels store it directly
    io = batch.io_stats()
    assert (io["d2h"], io["direct"]) == ((out.nbytes, 0) if mode == "always" else (0, out.nbytes)), io
    _close(out, c["out"], True)


def test_host_buffer_result_paths():
    """write_and_attend from host arrays: a page-locked result buffer (what the Python
    surface hands out) is stored into by the kernels, with no device-to-host copy; a pageable
    buffer through the C entry gets the copy; both equal the device-buffer result bit for bit."""
    torch = torch_cuda()
    from pagellm_b200 import _lib, workloads
    from pagellm_b200.cache import PagedBatch

    w = workloads.c2(3)
    pool = make_pool(w)
    q, k, v = dev_inputs(w)
    b = PagedBatch(pool, w.csr(), w.starts, w.n_new)
    ref = b.write_and_attend(0, q, k, v).cpu().numpy()  # re-appending equal rows is a no-op
    qh, kh, vh = q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy()
    got = b.write_and_attend(0, qh, kh, vh)
    assert b.io_stats() == {"h2d": qh.nbytes + kh.nbytes + vh.nbytes, "d2h": 0, "direct": qh.nbytes}
    np.testing.assert_array_equal(got, ref)
    # page-locked inputs travel by the one-launch gather instead of three copies: same bits
    qp, kp, vp = (torch.empty(t.shape, dtype=torch.float32, pin_memory=True) for t in (q, k, v))
    qp.copy_(q)
    kp.copy_(k)
    vp.copy_(v)
    got_pinned = b.write_and_attend(0, qp.numpy(), kp.numpy(), vp.numpy())
    assert b.io_stats()["h2d"] == qh.nbytes + kh.nbytes + vh.nbytes
    np.testing.assert_array_equal(got_pinned, ref)
    out = np.full_like(qh, np.nan)  # pageable
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.load().pk_batch_write_and_attend_host(b._b, 0, w.H, qh.ctypes.data, kh.ctypes.data,
                                                          vh.ctypes.data, out.ctypes.data, st))
    assert b.io_stats() == {"h2d": qh.nbytes + kh.nbytes + vh.nbytes, "d2h": qh.nbytes, "direct": 0}
    np.testing.assert_array_equal(out, ref)


def test_golden_paged_attention_cases():
    from pagellm_b200.cache import paged_attention

    z = load_npz("paged_attention_cases.npz")
    for ci in range(int(z["ncases"])):
        ctx, n, bs = (int(x) for x in z[f"c{ci}_meta"])
        got = paged_attention(z[f"c{ci}_q"], z[f"c{ci}_kp"], z[f"c{ci}_vp"],
                              z[f"c{ci}_table"].tolist(), ctx, ctx - n)
        assert got.dtype == np.float64
        np.testing.assert_allclose(got, z[f"c{ci}_paged"], rtol=F32_RTOL, atol=F32_ATOL)


def test_golden_batched_decode_garbage_padding():
    from pagellm_b200.cache import batched_decode_attention

    z = load_npz("batched_decode.npz")
    got = batched_decode_attention(z["q"], z["k"], z["v"], z["valid"])
    np.testing.assert_allclose(got, z["out"], rtol=F32_RTOL, atol=F32_ATOL)


def test_golden_slot_mapping():
    from pagellm_b200.cache import slot_mapping

    z = load_npz("slot_mapping.npz")
    for ci in range(int(z["ncases"])):
        got = slot_mapping(z[f"s{ci}_table"], z[f"s{ci}_pos"], int(z[f"s{ci}_bs"]))
        assert got.dtype == np.int64
        np.testing.assert_array_equal(got, z[f"s{ci}_slots"])


# ----------------------------------------------------------------------------- configs
def _run_config(w, check_seqs, seed=0):
    torch = torch_cuda()
    from pagellm_b200.cache import PagedBatch

    pool = make_pool(w, seed)
    if w.cow_pairs:
        src = np.array([p[0] for p in w.cow_pairs])
        before = pool.k[0, torch.as_tensor(src, device="cuda")].clone()
        pool.copy_blocks(w.cow_pairs)
        dst = torch.as_tensor(np.array([p[1] for p in w.cow_pairs]), device="cuda")
        assert torch.equal(pool.k[0, dst], before)
    batch = PagedBatch(pool, w.tables, w.starts, w.n_new)
    meta = po.StepMeta(w.tables, w.starts, w.n_new, w.bs)
    np.testing.assert_array_equal(batch.slots, meta.slots)
    np.testing.assert_array_equal(batch.positions, meta.positions)
    q, k, v = dev_inputs(w, seed + 1)
    out = batch.write_and_attend(0, q, k, v)
    batch.check()
    # append: pool rows at the step's slots hold k, v rounded to the pool dtype, bit-exact
    sl = torch.as_tensor(meta.slots, device="cuda")
    if w.dtype == "bf16":
        assert np.array_equal(bf16_bits_of_tensor(pool.k_flat[0].index_select(0, sl)),
                              po.bf16_bits(k.cpu().numpy()).reshape(k.shape))
        assert np.array_equal(bf16_bits_of_tensor(pool.v_flat[0].index_select(0, sl)),
                              po.bf16_bits(v.cpu().numpy()).reshape(v.shape))
    else:
        assert torch.equal(pool.k_flat[0].index_select(0, sl), k)
        assert torch.equal(pool.v_flat[0].index_select(0, sl), v)
    got = out.cpu().numpy()
    qh = q.cpu().numpy()
    for i, (rows, ref) in oracle_rows(pool, w, check_seqs, qh).items():
        _close(got[rows], ref, w.dtype == "bf16")
    assert np.isfinite(got).all()
    return pool, batch, got


def test_c1_full_fp32():
    from pagellm_b200 import workloads

    w = workloads.c1(0)
    _run_config(w, range(w.nseq))


def test_c2_llama8b_decode_bf16():
    from pagellm_b200 import workloads

    w = workloads.c2(0)
    pool, batch, _ = _run_config(w, range(w.nseq))
    assert pool.tensor_core_path[0], pool.tensor_core_path[1]
    st = batch.stats()
    assert st["tc_units"] == w.nseq and st["generic_rows"] == 0 and st["tc_ctas"] > 0


def test_c2_split_units_merge():
    """Two long sequences over ~150 CTAs: every unit is cut across many CTAs, so the
    partial (max, sum, output) merge carries the whole result."""
    from pagellm_b200 import workloads

    w = workloads.c2(3, batch=2)
    _, batch, _ = _run_config(w, [0, 1])
    assert batch.stats()["split_units"] == 2


def test_c3_mixed_chunked_prefill():
    from pagellm_b200 import workloads

    w = workloads.c3(0)
    _run_config(w, range(w.nseq))


def test_c4_prefix_sharing_cow_verify():
    from pagellm_b200 import workloads

    w = workloads.c4(0)
    assert len(w.cow_pairs) == 192
    _run_config(w, range(w.nseq))


def test_c5_full_batch_and_head_shards():
    """The whole 128-sequence C5 batch (~1.4M context tokens) on one pool against the oracle
    on every row; then the head-sharded layout at its 2-GPU and 8-GPU shard sizes (4 and 1 KV
    heads per pool, the pool's head slice copied out of the full pool): every shard's output
    against the same oracle rows, restricted to its query heads."""
    torch = torch_cuda()
    from pagellm_b200 import workloads
    from pagellm_b200.cache import PagedBatch

    w = workloads.c5(0)
    assert w.nseq == 128
    pool, _, got = _run_config(w, [])
    q, k, v = dev_inputs(w, 1)
    qh = q.cpu().numpy()
    ref = np.empty_like(got)
    for i, (rows, r) in oracle_rows(pool, w, range(w.nseq), qh).items():
        ref[rows] = r
    _close(got, ref, True)
    g = w.H // w.KVH
    for kh, heads in ((4, (0, 4)), (1, (0, 5))):
        part = workloads.c5(0, kv_heads=kh)
        sp = make_pool(part, 0)
        for h0 in heads:
            sp.k_flat[0].copy_(pool.k_flat[0][:, h0:h0 + kh])
            sp.v_flat[0].copy_(pool.v_flat[0][:, h0:h0 + kh])
            qs = q[:, h0 * g:(h0 + kh) * g].contiguous()
            ks, vs = k[:, h0:h0 + kh].contiguous(), v[:, h0:h0 + kh].contiguous()
            b = PagedBatch(sp, part.tables, part.starts, part.n_new)
            o = b.write_and_attend(0, qs, ks, vs).cpu().numpy()
            b.check()
            _close(o, ref[:, h0 * g:(h0 + kh) * g], True)
        del sp
        torch.cuda.empty_cache()


@pytest.mark.parametrize("D,KVH,g", [(64, 1, 8), (64, 2, 8), (256, 1, 4), (256, 2, 4)])
def test_few_kv_heads_virtual_ctas(D, KVH, g):
    """Pools of 1-2 KV heads (head-sharded shards) run V = 8/kvh virtual CTAs per CTA, each with
    its own block range and stage ring (fewer at head_dim 256, where shared memory runs out):
    a decode step of 24 long sequences, every row against the oracle, append bit-exact."""
    from pagellm_b200 import workloads

    rng = np.random.default_rng(D * 10 + KVH)
    L = rng.integers(200, 3000, size=24).astype(np.int64)
    need = int(sum(-(-int(x) // 16) for x in L))
    nb = int(np.ceil(1.25 * need))
    tables = workloads._scatter_tables(rng, L, 16, nb)
    w = workloads.Workload("fewkv", g * KVH, KVH, D, 16, "bf16", nb, tables, (L - 1).astype(np.int64),
                           np.ones(len(L), np.int64))
    pool, batch, _ = _run_config(w, range(w.nseq))
    assert pool.tensor_core_path[0], pool.tensor_core_path[1]
    assert batch.stats()["split_units"] > 0


# ----------------------------------------------------------------------------- bit-exact ops
def test_copy_blocks_bit_exact_and_ordered():
    torch = torch_cuda()
    from pagellm_b200 import workloads

    w = workloads.c2(1, batch=4)
    pool = make_pool(w, 5, layers=2)
    kh = pool.k.float().cpu().numpy()
    vh = pool.v.float().cpu().numpy()
    # 3 -> 7 then 7 -> 9 must see the copied data (list order), 1 -> 2 independent
    pairs = [(3, 7), (1, 2), (7, 9), (11, 3)]
    po.copy_blocks(kh, vh, pairs)
    pool.copy_blocks(pairs)
    torch.cuda.synchronize()
    assert np.array_equal(pool.k.float().cpu().numpy(), kh)
    assert np.array_equal(pool.v.float().cpu().numpy(), vh)
    with pytest.raises(IndexError):
        pool.copy_blocks([(0, w.num_blocks)])


def test_fp32_pool_append_exact():
    torch = torch_cuda()
    from pagellm_b200 import workloads
    from pagellm_b200.cache import PagedBatch

    w = workloads.c1(2)
    pool = make_pool(w, 3, layers=3)
    q, k, v = dev_inputs(w, 4)
    b = PagedBatch(pool, w.tables, w.starts, w.n_new)
    b.write_and_attend(2, q, k, v)
    sl = torch.as_tensor(b.slots, device="cuda")
    assert torch.equal(pool.k_flat[2].index_select(0, sl), k)
    assert torch.equal(pool.v_flat[2].index_select(0, sl), v)


@pytest.mark.parametrize("D,dt", [(32, "bfloat16"), (96, "bfloat16"), (192, "bfloat16"), (16, np.float32),
                                  (48, np.float32)])
def test_cuda_core_path_appends_in_kernel(D, dt):
    """Head sizes the tensor-core kernel does not take run on the CUDA-core kernels, which
    append the step's rows inside the attention launch (lanes over keys at head_dim <= 32,
    over dimensions above). head_dim 192 is a multiple of 64 without a tensor-core instance:
    a bf16 pool of that size must land here too, not on the tensor-core launch. The pool holds the rows exactly as the append kernel would
    write them (bf16: round to nearest even), the output matches the oracle on the pool's
    contents, and the step is one launch; decode rows and multi-token rows are mixed."""
    torch = torch_cuda()
    from pagellm_b200.cache import PagedBatch, PagedKVPool

    bf = dt == "bfloat16"
    H, KVH, bs, nb = 8, 2, 16, 64
    pool = PagedKVPool(Shape(1, KVH, D), nb, bs, dt)
    assert not pool.tensor_core_path[0]
    g = torch.Generator(device="cuda").manual_seed(D)
    pool.k.copy_(torch.randn(pool.k.shape, generator=g, device="cuda").to(pool.k.dtype))
    pool.v.copy_(torch.randn(pool.v.shape, generator=g, device="cuda").to(pool.v.dtype))
    ctx = [1, 16, 33, 70, 5, 129]
    n_new = [1, 1, 4, 2, 5, 1]
    perm = np.random.default_rng(D).permutation(nb)
    tables, used = [], 0
    for c_ in ctx:
        n = -(-c_ // bs)
        tables.append(perm[used:used + n].tolist())
        used += n
    starts = [c_ - n for c_, n in zip(ctx, n_new)]
    b = PagedBatch(pool, tables, starts, n_new)
    rows = sum(n_new)
    q = torch.randn((rows, H, D), generator=g, device="cuda")
    k = torch.randn((rows, KVH, D), generator=g, device="cuda")
    v = torch.randn((rows, KVH, D), generator=g, device="cuda")
    out = b.write_and_attend(0, q, k, v).cpu().numpy()
    b.check()
    st = b.stats()
    assert st["generic_rows"] == rows and st["tc_units"] == 0 and st["launches"] == 1, st
    sl = torch.as_tensor(b.slots, device="cuda")
    if bf:
        assert np.array_equal(bf16_bits_of_tensor(pool.k_flat[0].index_select(0, sl)),
                              bf16_bits_of_tensor(k.to(torch.bfloat16)))
        assert np.array_equal(bf16_bits_of_tensor(pool.v_flat[0].index_select(0, sl)),
                              bf16_bits_of_tensor(v.to(torch.bfloat16)))
    else:
        assert torch.equal(pool.k_flat[0].index_select(0, sl), k)
        assert torch.equal(pool.v_flat[0].index_select(0, sl), v)
    meta = po.StepMeta(tables, starts, n_new, bs)
    qh = q.cpu().numpy()
    for i in range(len(ctx)):
        kc, vc = gather_rows(pool, 0, meta.ctx_slots[i])
        a, z = meta.offsets[i], meta.offsets[i + 1]
        _close(out[a:z], po.attention_dense(qh[a:z], kc, vc, starts[i]), bf)


# ----------------------------------------------------------------------------- edges
def test_edge_cases_context_lengths():
    """ctx 1, block-aligned contexts, a zero-row sequence and mixed window sizes."""
    torch = torch_cuda()
    from pagellm_b200.cache import PagedBatch, PagedKVPool

    for dt, bf in ((np.float32, False), ("bfloat16", True)):
        pool = PagedKVPool(Shape(1, 8, 128), 64, 16, dt)
        g = torch.Generator(device="cuda").manual_seed(0)
        pool.k.copy_(torch.randn(pool.k.shape, generator=g, device="cuda").to(pool.k.dtype))
        pool.v.copy_(torch.randn(pool.v.shape, generator=g, device="cuda").to(pool.v.dtype))
        ctx = [1, 16, 32, 17, 40, 7, 64]
        n_new = [1, 1, 16, 1, 0, 3, 9]
        perm = np.random.default_rng(0).permutation(64)
        tables, used = [], 0
        for c_ in ctx:
            nb = -(-c_ // 16)
            tables.append(perm[used:used + nb].tolist())
            used += nb
        starts = [c_ - n for c_, n in zip(ctx, n_new)]
        b = PagedBatch(pool, tables, starts, n_new)
        rows = sum(n_new)
        q = torch.randn((rows, 32, 128), device="cuda")
        k = torch.randn((rows, 8, 128), device="cuda")
        v = torch.randn((rows, 8, 128), device="cuda")
        out = b.write_and_attend(0, q, k, v).cpu().numpy()
        meta = po.StepMeta(tables, starts, n_new, 16)
        qh = q.cpu().numpy()
        for i in range(len(ctx)):
            if n_new[i] == 0:
                continue
            kc, vc = gather_rows(pool, 0, meta.ctx_slots[i])
            a, z = meta.offsets[i], meta.offsets[i + 1]
            _close(out[a:z], po.attention_dense(qh[a:z], kc, vc, starts[i]), bf)


def test_empty_batch_and_errors():
    torch = torch_cuda()
    from pagellm_b200.cache import PagedBatch, PagedKVPool

    pool = PagedKVPool(Shape(2, 2, 32), 8, 16)
    b = PagedBatch(pool, [], [], [])
    out = b.write_and_attend(0, np.zeros((0, 4, 32), np.float32), np.zeros((0, 2, 32), np.float32),
                             np.zeros((0, 2, 32), np.float32))
    assert out.shape == (0, 4, 32)
    with pytest.raises(IndexError):  # table too short for position 16
        PagedBatch(pool, [[0]], [16], [1])
    with pytest.raises(IndexError):  # block id outside the pool
        PagedBatch(pool, [[8]], [0], [1])
    with pytest.raises(IndexError):
        PagedBatch(pool, [[-1]], [0], [1])
    with pytest.raises(ValueError):
        PagedBatch(pool, [[0]], [0], [1], attn="flash")
    b = PagedBatch(pool, [[0]], [0], [1])
    with pytest.raises(ValueError):  # 3 query heads is not a multiple of 2 KV heads
        b.write_and_attend(0, np.zeros((1, 3, 32), np.float32), np.zeros((1, 2, 32), np.float32),
                           np.zeros((1, 2, 32), np.float32))
    with pytest.raises(IndexError):
        b.write_and_attend(2, np.zeros((1, 4, 32), np.float32), np.zeros((1, 2, 32), np.float32),
                           np.zeros((1, 2, 32), np.float32))
    torch.cuda.synchronize()


def test_decode_loop_reuses_batch_handles():
    """Ten decode steps through fresh PagedBatch objects: handles are recycled, and each
    step matches the oracle on the cache the previous steps built."""
    torch = torch_cuda()
    from pagellm_b200 import workloads
    from pagellm_b200.cache import PagedBatch

    w = workloads.c2(4, batch=6)
    pool = make_pool(w, 0)
    starts = w.starts.copy()
    spare = sorted(set(range(w.num_blocks)) - set(np.concatenate(w.tables).tolist()))
    tables = [np.concatenate([t, [spare[i]]]).astype(np.int32) for i, t in enumerate(w.tables)]
    for step in range(10):
        b = PagedBatch(pool, tables, starts, w.n_new)
        q = torch.randn((w.nseq, w.H, w.D), device="cuda")
        k = torch.randn((w.nseq, w.KVH, w.D), device="cuda")
        v = torch.randn((w.nseq, w.KVH, w.D), device="cuda")
        out = b.write_and_attend(0, q, k, v).cpu().numpy()
        meta = po.StepMeta(tables, starts, w.n_new, w.bs)
        for i in range(w.nseq):
            kc, vc = gather_rows(pool, 0, meta.ctx_slots[i])
            _close(out[i:i + 1], po.attention_dense(q.cpu().numpy()[i:i + 1], kc, vc, int(starts[i])), True)
        starts = starts + 1
    assert len(pool._idle_batches) <= 2


def test_shared_and_repeated_written_blocks_follow_pagellm():
    """Outside what BlockManager produces: two sequences write the same slot of a shared
    block, a sequence reads that shared block, and a table repeats a block id. pagellm's
    numpy semantics - all rows appended first, last writer of a slot wins, then attention
    reads the pool - hold exactly (the step falls back to the separate append kernel)."""
    torch = torch_cuda()
    from pagellm_b200.cache import PagedBatch, PagedKVPool

    pool = PagedKVPool(Shape(1, 8, 128), 16, 16, "bfloat16")
    g = torch.Generator(device="cuda").manual_seed(3)
    pool.k.copy_(torch.randn(pool.k.shape, generator=g, device="cuda").to(pool.k.dtype))
    pool.v.copy_(torch.randn(pool.v.shape, generator=g, device="cuda").to(pool.v.dtype))
    tables = [[0, 1], [2, 1], [3, 4], [5, 5]]
    starts = [19, 19, 31, 29]
    n_new = [1, 1, 1, 1]
    rng = np.random.default_rng(0)
    q = rng.standard_normal((4, 32, 128), dtype=np.float32)
    k = po.bf16_round(rng.standard_normal((4, 8, 128), dtype=np.float32))
    v = po.bf16_round(rng.standard_normal((4, 8, 128), dtype=np.float32))
    kf = pool.k_flat[0].float().cpu().numpy()
    vf = pool.v_flat[0].float().cpu().numpy()
    meta = po.StepMeta(tables, starts, n_new, 16)
    ref = po.write_and_attend(kf, vf, meta, q, k, v)
    b = PagedBatch(pool, tables, starts, n_new)
    out = b.write_and_attend(0, q, k, v)
    assert b.stats()["launches"] >= 2  # append kernel ran on its own
    np.testing.assert_array_equal(pool.k_flat[0].float().cpu().numpy(), kf)
    np.testing.assert_array_equal(pool.v_flat[0].float().cpu().numpy(), vf)
    _close(out, ref, True)


def test_fused_append_single_launch_c2():
    """The common case: private written blocks -> one kernel launch per layer (append
    and partial merge folded into the attention kernel)."""
    from pagellm_b200 import workloads
    from pagellm_b200.cache import PagedBatch

    w = workloads.c2(5, batch=16)
    pool = make_pool(w, 0)
    q, k, v = dev_inputs(w, 2)
    b = PagedBatch(pool, w.tables, w.starts, w.n_new)
    b.write_and_attend(0, q, k, v)
    st = b.stats()
    assert st["launches"] == 1 and st["split_units"] > 0


@pytest.mark.parametrize("H,KVH,bs", [(32, 8, 16), (64, 8, 16), (16, 4, 32), (8, 8, 16), (16, 1, 64)])
def test_wide_tile_chunks_match_oracle(H, KVH, bs):
    """Chunked prefill / long verify windows on the tcgen05 wide-tile kernel: prefill from
    position 0, chunks over a cached prefix with lengths off the 128-row tile, next to
    decode rows (split-KV kernel) in one step."""
    torch = torch_cuda()
    from pagellm_b200.cache import PagedBatch, PagedKVPool

    g = H // KVH
    ctx = [100, 1536, 333, 57, 900, 64]
    n_new = [100, 512, 48, 1, 1, 20]
    nb = sum(-(-c // bs) for c in ctx) + 8
    rng = np.random.default_rng(H + bs)
    perm = rng.permutation(nb)
    tables, used = [], 0
    for c in ctx:
        k_ = -(-c // bs)
        tables.append(perm[used:used + k_].tolist())
        used += k_
    starts = [c - n for c, n in zip(ctx, n_new)]
    pool = PagedKVPool(Shape(1, KVH, 128), nb, bs, "bfloat16")
    gen = torch.Generator(device="cuda").manual_seed(9)
    pool.k.copy_(torch.randn(pool.k.shape, generator=gen, device="cuda").to(pool.k.dtype))
    pool.v.copy_(torch.randn(pool.v.shape, generator=gen, device="cuda").to(pool.v.dtype))
    rows = sum(n_new)
    q = torch.randn((rows, H, 128), generator=gen, device="cuda")
    k = torch.randn((rows, KVH, 128), generator=gen, device="cuda")
    v = torch.randn((rows, KVH, 128), generator=gen, device="cuda")
    b = PagedBatch(pool, tables, starts, n_new)
    out = b.write_and_attend(0, q, k, v)
    b.check()
    st = b.stats()
    assert st["wide_items"] > 0, st
    got, qh = out.cpu().numpy(), q.cpu().numpy()
    meta = po.StepMeta(tables, starts, n_new, bs)
    for i in range(len(ctx)):
        kc, vc = gather_rows(pool, 0, meta.ctx_slots[i])
        a, z = meta.offsets[i], meta.offsets[i + 1]
        _close(got[a:z], po.attention_dense(qh[a:z], kc, vc, starts[i]), True)
    # the appended rows of every sequence (wide and split-KV) are in the pool, bit for bit
    sl = torch.as_tensor(meta.slots, device="cuda")
    assert np.array_equal(bf16_bits_of_tensor(pool.k_flat[0].index_select(0, sl)),
                          po.bf16_bits(k.cpu().numpy()).reshape(k.shape))


@pytest.mark.parametrize("mode", ["auto", "always", "off"])
def test_shared_prefix_forks_match_oracle(mode):
    """C4's shape at 4 requests: 16 forks over one ref-counted 2048-token prefix, CoW'd
    partial blocks, 5 verify tokens each. With prefix sharing the shared blocks are
    attended once per 128 rows (tcgen05 kernel) and merged with the split-KV result for the
    rest of each fork; every mode matches the oracle."""
    torch = torch_cuda()
    from pagellm_b200 import workloads
    from pagellm_b200.cache import PagedBatch

    w = workloads.c4(2, requests=4)
    pool = make_pool(w, 0)
    pool.copy_blocks(w.cow_pairs)
    b = PagedBatch(pool, w.tables, w.starts, w.n_new)
    b.prefix_sharing = mode
    assert b.prefix_sharing == mode
    q, k, v = dev_inputs(w, 1)
    out = b.write_and_attend(0, q, k, v)
    b.check()
    ps = b.prefix_stats()
    if mode == "off":
        assert ps == {"groups": 0, "items": 0, "shared_keys": 0, "token_keys": 0}
    else:
        # 16 forks x 5 tokens x g=4 rows = 320 rows -> 3 items of 128 rows
        assert ps == {"groups": 1, "items": 3, "shared_keys": 2048, "token_keys": 80 * 2048}, ps
    got, qh = out.cpu().numpy(), q.cpu().numpy()
    for i, (rows, ref) in oracle_rows(pool, w, range(w.nseq), qh).items():
        _close(got[rows], ref, True)
    torch.cuda.synchronize()


@pytest.mark.parametrize("H,KVH,bs", [(32, 8, 16), (64, 8, 16), (16, 4, 32), (8, 8, 16), (16, 1, 64)])
def test_shared_prefix_groups_mixed_step(H, KVH, bs):
    """Several prefix groups in one step beside unshared decode rows and a prefill chunk:
    prefixes off block boundaries, one member whose first new token lies inside the shared
    blocks (so the group's prefix is cut there, and its append writes a block the others
    read), members with 1..7 new tokens; compared with the oracle and with sharing off."""
    torch = torch_cuda()
    from pagellm_b200.cache import PagedBatch, PagedKVPool

    rng = np.random.default_rng(H * 7 + bs)
    # (shared prefix tokens, [(start, n_new), ...]); solo sequences have prefix 0
    spec = [(700, [(705, 1), (709, 5), (700 + bs, 3), (701, 1), (760, 7)]),
            (4 * bs, [(4 * bs + 3, 2), (4 * bs, 4)]),
            (300, [(320, 1), (330, 1), (100, 2)]),
            (0, [(499, 1)]), (0, [(1000, 200)]), (0, [(37, 3)])]
    tables, starts, n_new, need = [], [], [], 0
    for pre, mem in spec:
        need += pre // bs + sum(-(-(st + n) // bs) for st, n in mem)
    nb = need + 16
    perm = iter(rng.permutation(nb).tolist())
    for pre, mem in spec:
        shared = [next(perm) for _ in range(pre // bs)]
        for st, n in mem:
            own = -(-(st + n) // bs) - len(shared)
            tables.append(shared + [next(perm) for _ in range(max(own, 0))])
            starts.append(st)
            n_new.append(n)
    pool = PagedKVPool(Shape(1, KVH, 128), nb, bs, "bfloat16")
    gen = torch.Generator(device="cuda").manual_seed(5)
    pool.k.copy_(torch.randn(pool.k.shape, generator=gen, device="cuda").to(pool.k.dtype))
    pool.v.copy_(torch.randn(pool.v.shape, generator=gen, device="cuda").to(pool.v.dtype))
    k0, v0 = pool.k.clone(), pool.v.clone()
    rows = sum(n_new)
    q = torch.randn((rows, H, 128), generator=gen, device="cuda")
    k = torch.randn((rows, KVH, 128), generator=gen, device="cuda")
    v = torch.randn((rows, KVH, 128), generator=gen, device="cuda")
    outs = {}
    for mode in ("always", "off"):
        pool.k.copy_(k0)
        pool.v.copy_(v0)
        b = PagedBatch(pool, tables, starts, n_new)
        b.prefix_sharing = mode
        outs[mode] = b.write_and_attend(0, q, k, v).cpu().numpy()
        b.check()
        ps = b.prefix_stats()
        if mode == "always":
            # a member with n_new * g >= 64 query rows takes the wide chunk path and leaves
            # its group; a group needs two members left; its prefix is cut at the first
            # block holding any remaining member's first new token (group 3: the member at 100)
            g = H // KVH
            groups = keys = 0
            for pre, mem in spec:
                left = [st for st, n in mem if n * g < 64]
                if pre and len(left) >= 2:
                    groups += 1
                    keys += min([pre // bs] + [st // bs for st in left]) * bs
            assert ps["groups"] == groups and ps["shared_keys"] == keys, ps
            assert groups >= 2
            assert b.stats()["wide_items"] > 0
    qh = q.cpu().numpy()
    meta = po.StepMeta(tables, starts, n_new, bs)
    for i in range(len(tables)):
        kc, vc = gather_rows(pool, 0, meta.ctx_slots[i])
        a, z = meta.offsets[i], meta.offsets[i + 1]
        ref = po.attention_dense(qh[a:z], kc, vc, starts[i])
        _close(outs["always"][a:z], ref, True)
        _close(outs["off"][a:z], ref, True)
    # both schedules agree far more closely than the bf16 tolerance
    assert float(np.max(np.abs(outs["always"] - outs["off"]))) < 5e-3


def test_speculative_rollback_on_the_paged_pool():
    """Verify 5 draft tokens, keep 2 (BlockManager.truncate), decode the next token: it sees
    exactly the 23 kept positions; the rejected drafts' K/V left in the kept block are
    neither attended nor leaked, and the new token overwrites the first rejected slot."""
    torch = torch_cuda()
    from pagellm_b200.cache import BlockManager, PagedBatch, PagedKVPool

    H, KVH, bs = 8, 2, 16
    bm = BlockManager(32, bs)
    pool = PagedKVPool(Shape(1, KVH, 128), 32, bs, "bfloat16")
    gen = torch.Generator(device="cuda").manual_seed(11)
    prompt = list(range(20))
    bm.allocate(0, prompt)

    def step(start, n):
        bm.ensure_capacity(0, start + n, write_from=start)
        q = torch.randn((n, H, 128), generator=gen, device="cuda")
        k = torch.randn((n, KVH, 128), generator=gen, device="cuda")
        v = torch.randn((n, KVH, 128), generator=gen, device="cuda")
        b = PagedBatch(pool, [bm.block_table(0)], [start], [n])
        out = b.write_and_attend(0, q, k, v)
        b.check()
        return q, out

    step(0, 20)                  # prefill
    step(20, 5)                  # verify window: drafts at 20..24
    bm.truncate(0, 22)           # 2 accepted
    assert len(bm.block_table(0)) == 2
    q, out = step(22, 1)         # next token lands at 22
    slots = po.slot_mapping(bm.block_table(0), np.arange(23), bs)
    kc, vc = gather_rows(pool, 0, slots)
    _close(out.cpu().numpy(), po.attention_dense(q.cpu().numpy(), kc, vc, 22), True)


def test_injected_launch_failure_raises_and_batch_recovers():
    """Fault injection on the host (a test hook in the library, no GPU fault): the next
    attention call fails as a launch error would, raises, and leaves the batch usable."""
    from pagellm_b200 import _lib, workloads
    from pagellm_b200.cache import PagedBatch

    w = workloads.c2(1, batch=4)
    pool = make_pool(w, 0)
    b = PagedBatch(pool, w.tables, w.starts, w.n_new)
    q, k, v = dev_inputs(w, 1)
    assert _lib.load().pk_test_inject_launch_failure() == 0
    with pytest.raises(RuntimeError, match="injected"):
        b.write_and_attend(0, q, k, v)
    out = b.write_and_attend(0, q, k, v)  # nothing was appended by the failed call
    b.check()
    got, qh = out.cpu().numpy(), q.cpu().numpy()
    for i, (rows, ref) in oracle_rows(pool, w, range(w.nseq), qh).items():
        _close(got[rows], ref, True)


def test_bounded_wait_gives_up_and_context_survives():
    """Failure detection without a GPU fault: a wait on a barrier phase that nothing
    completes returns after its limit with an error status the host reads; the context
    is still usable afterwards."""
    import ctypes as C
    import time

    torch = torch_cuda()
    from pagellm_b200 import _lib, workloads

    lib = _lib.load()
    flag = C.c_int(-1)
    t0 = time.perf_counter()
    assert lib.pk_selftest_bounded_wait(0, 50_000_000, C.byref(flag)) == 0, _lib.last_error()
    assert flag.value == 1
    assert time.perf_counter() - t0 < 10.0
    w = workloads.c2(2, batch=3)
    _run_config(w, range(w.nseq))
    torch.cuda.synchronize()
