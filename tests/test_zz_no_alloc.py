"""The decode-attention entry point that allocates nothing (pk_decode_attend_static).

Some callers cannot call cudaMalloc: a serving framework that owns all of HBM through its
own caching allocator, or a plugin host that bans cudaMalloc / cudaFree on the request path
(cudaFree synchronises the whole device). pk_decode_attend_static serves them: its scratch
is a fixed 16 MiB device array inside the library. These tests call it through the C ABI
and compare it, on two calls in a row, with the regular entry point (pk_batch_plan +
pk_batch_attend) and with the CPU oracle on every output row, within the bf16 tolerance the
other GPU tests use.

This file is collected last on purpose: a run that stops at its first failure has run
every other test before it reaches these.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oracle import paged_oracle as po

pytestmark = pytest.mark.gpu

BF16_ATOL = 2e-2


class _Shape:
    def __init__(self, n_layers, n_kv_heads, head_dim):
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim


def _filled_pool(shape, num_blocks, bs, seed):
    import torch

    from pagellm_b200.cache import PagedKVPool

    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    pool = PagedKVPool(shape, num_blocks, bs, "bfloat16")
    g = torch.Generator(device="cuda").manual_seed(seed)
    for t in (pool.k, pool.v):
        t.copy_(torch.randn(t.shape, generator=g, device="cuda").to(t.dtype))
    return pool


def _static_call(lib, pool, H, tables, ctx, layer, q, out, err):
    import torch

    lens = np.array([len(t) for t in tables], np.int64)
    indptr = np.zeros(len(tables) + 1, np.int64)
    np.cumsum(lens, out=indptr[1:])
    ids = np.ascontiguousarray(np.concatenate([np.asarray(t, np.int32) for t in tables]))
    ctx = np.ascontiguousarray(ctx, dtype=np.int64)
    return lib.pk_decode_attend_static(
        pool.handle, layer, H, len(tables),
        indptr.ctypes.data_as(C.POINTER(C.c_int64)), ids.ctypes.data_as(C.POINTER(C.c_int32)),
        ctx.ctypes.data_as(C.POINTER(C.c_int64)), q.data_ptr(), out.data_ptr(),
        err.data_ptr() if err is not None else None, torch.cuda.current_stream().cuda_stream)


def _oracle_max_err(pool, layer, tables, ctx, q, out, bs):
    """Largest |out - oracle| over every row: the oracle reads the device pool's bf16 K/V
    widened to float32, each row at position ctx-1 over positions 0..ctx-1."""
    import torch

    qh, got = q.cpu().numpy(), out.cpu().numpy()
    worst = 0.0
    for i, (t, L) in enumerate(zip(tables, ctx)):
        slots = torch.as_tensor(po.slot_mapping(t, np.arange(int(L)), bs), device=pool.device)
        kc = pool.k_flat[layer].index_select(0, slots).float().cpu().numpy()
        vc = pool.v_flat[layer].index_select(0, slots).float().cpu().numpy()
        ref = po.attention_dense(qh[i:i + 1], kc, vc, int(L) - 1)
        worst = max(worst, float(np.max(np.abs(got[i:i + 1] - ref))))
    return worst


def _check_two_calls(pool, H, tables, ctx, bs, layers, seed):
    """Two calls in a row (different layers and inputs): static entry == regular entry
    within the bf16 tolerance, and == the oracle on every row."""
    import torch

    from pagellm_b200 import _lib
    from pagellm_b200.cache import PagedBatch

    lib = _lib.load()
    batch = PagedBatch(pool, tables, [int(L) - 1 for L in ctx], [1] * len(tables))
    assert batch.stats()["rows"] == len(tables)
    g = torch.Generator(device="cuda").manual_seed(seed)
    for layer in layers:
        q = torch.randn((len(tables), H, pool.head_dim), generator=g, device="cuda")
        ref = batch.attend(layer, q)
        out = torch.full_like(q, float("nan"))
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        rc = _static_call(lib, pool, H, tables, ctx, layer, q, out, err)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.isfinite(out).all()
        diff = float((out - ref).abs().max())
        assert diff <= BF16_ATOL, diff
        worst = _oracle_max_err(pool, layer, tables, ctx, q, out, bs)
        assert worst <= BF16_ATOL, worst


def test_static_entry_matches_batch_entry_twice():
    """C2's shape (8 KV heads, head_dim 128, 16-token blocks, g = 4) at 48 sequences."""
    from pagellm_b200 import workloads

    w = workloads.c2(11, batch=48)
    pool = _filled_pool(_Shape(2, w.KVH, w.D), w.num_blocks, w.bs, 11)
    _check_two_calls(pool, w.H, w.tables, w.ctx_lens, w.bs, (1, 0), 5)


@pytest.mark.parametrize("D,KVH,H", [(64, 8, 32), (128, 8, 64), (256, 4, 16)])
def test_static_entry_split_sequences(D, KVH, H):
    """Three long sequences over the whole GPU: every one is cut across many CTAs, so the
    result comes from the separate partial-merge launch the static entry uses (the regular
    entry merges inside the attention kernel). Head sizes 64 / 128 / 256 and g = 4 / 8 / 4."""
    bs = 16
    ctx = [3001, 2048, 777]
    nblk = [-(-L // bs) for L in ctx]
    nb = sum(nblk) + 5
    perm = np.random.default_rng(D).permutation(nb).astype(np.int32)
    tables, used = [], 0
    for n in nblk:
        tables.append(perm[used:used + n])
        used += n
    pool = _filled_pool(_Shape(2, KVH, D), nb, bs, D)
    assert pool.tensor_core_path[0], pool.tensor_core_path[1]
    _check_two_calls(pool, H, tables, ctx, bs, (0, 1), D + 1)


def test_static_entry_rejects_oversize_and_missing_error_word_before_launch():
    import torch

    from pagellm_b200 import _lib, workloads

    lib = _lib.load()
    w = workloads.c2(12, batch=4)
    pool = _filled_pool(_Shape(1, w.KVH, w.D), w.num_blocks, w.bs, 12)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    q = torch.zeros((600, w.H, w.D), device="cuda")
    out = torch.zeros_like(q)
    tables = [np.zeros(1, np.int32)] * 600
    rc = _static_call(lib, pool, w.H, tables, np.ones(600, np.int64), 0, q, out, err)
    assert rc == _lib.PK_ERR_INVALID_ARG
    assert "static scratch" in _lib.last_error()
    # a plan larger than the 16 MiB array: 512 one-block sequences still need
    # (512 + CTAs) x 8 heads x 16 columns x 128 dims of float partials (> 40 MB)
    bp = _filled_pool(_Shape(1, 8, 128), 512, 16, 1)
    tables = [np.array([i], np.int32) for i in range(512)]
    qb = torch.zeros((512, 32, 128), device="cuda")
    ob = torch.zeros_like(qb)
    rc = _static_call(lib, bp, 32, tables, np.full(512, 16, np.int64), 0, qb, ob, err)
    assert rc == _lib.PK_ERR_INVALID_ARG
    assert "scratch" in _lib.last_error()
    # without an error word a timed-out wait could not be reported: refused
    tables = w.tables
    q4 = torch.zeros((w.nseq, w.H, w.D), device="cuda")
    o4 = torch.zeros_like(q4)
    rc = _static_call(lib, pool, w.H, tables, w.ctx_lens, 0, q4, o4, None)
    assert rc == _lib.PK_ERR_INVALID_ARG
    assert "err_dev" in _lib.last_error()
    torch.cuda.synchronize()
    assert float(ob.abs().max()) == 0.0 and float(o4.abs().max()) == 0.0  # nothing was launched
    assert int(err.item()) == 0


def test_static_entry_refuses_stream_capture():
    """The call uploads from its own host memory, which a graph replay would read after it is
    gone: on a capturing stream it returns PK_ERR_UNSUPPORTED and enqueues nothing."""
    import torch

    from pagellm_b200 import _lib, workloads

    lib = _lib.load()
    w = workloads.c2(13, batch=4)
    pool = _filled_pool(_Shape(1, w.KVH, w.D), w.num_blocks, w.bs, 13)
    q = torch.randn((w.nseq, w.H, w.D), device="cuda")
    out = torch.zeros_like(q)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _static_call(lib, pool, w.H, w.tables, w.ctx_lens, 0, q, out, err) == 0  # eager: fine
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    rc = None
    with torch.cuda.stream(side):
        graph.capture_begin()
        try:
            rc = _static_call(lib, pool, w.H, w.tables, w.ctx_lens, 0, q, out, err)
            marker = out.sum()  # something for the graph to hold
        finally:
            graph.capture_end()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    assert rc == _lib.PK_ERR_UNSUPPORTED
    assert "graph" in _lib.last_error()
    del marker, graph
