"""The decode-attention entry point that allocates nothing (pk_decode_attend_static).

Some callers cannot call cudaMalloc: a serving framework that owns all of HBM through its
own caching allocator, or a plugin host that bans cudaMalloc / cudaFree on the request path
(cudaFree synchronises the whole device). pk_decode_attend_static serves them: its scratch
is a fixed 16 MiB device array inside the library. These tests call it through the C ABI
and compare it with the regular entry point (pk_batch_plan + pk_batch_attend), within the
bf16 tolerance the other GPU tests use, on two calls in a row.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BF16_ATOL = 2e-2


def _setup(seed: int, batch: int):
    import torch

    from pagellm_b200 import workloads
    from pagellm_b200.cache import PagedKVPool

    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    w = workloads.c2(seed, batch=batch)

    class Shape:
        n_layers, n_kv_heads, head_dim = 2, w.KVH, w.D

    pool = PagedKVPool(Shape, w.num_blocks, w.bs, "bfloat16")
    g = torch.Generator(device="cuda").manual_seed(seed)
    for t in (pool.k, pool.v):
        t.copy_(torch.randn(t.shape, generator=g, device="cuda").to(t.dtype))
    return w, pool


def _static_call(lib, pool, w, layer, q, out):
    import torch

    indptr, ids = w.csr()
    ctx = np.ascontiguousarray(w.ctx_lens, dtype=np.int64)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.pk_decode_attend_static(
        pool.handle, layer, w.H, w.nseq,
        indptr.ctypes.data_as(C.POINTER(C.c_int64)), ids.ctypes.data_as(C.POINTER(C.c_int32)),
        ctx.ctypes.data_as(C.POINTER(C.c_int64)), q.data_ptr(), out.data_ptr(), err.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    return rc, err


def test_static_entry_matches_batch_entry_twice():
    import torch

    from pagellm_b200 import _lib
    from pagellm_b200.cache import PagedBatch

    lib = _lib.load()
    w, pool = _setup(11, 48)
    batch = PagedBatch(pool, w.tables, w.starts, w.n_new)  # decode rows at ctx-1
    assert batch.stats()["rows"] == w.nseq
    g = torch.Generator(device="cuda").manual_seed(5)
    for layer in (1, 0):  # two calls in a row, different inputs
        q = torch.randn((w.nseq, w.H, w.D), generator=g, device="cuda")
        ref = batch.attend(layer, q)
        out = torch.full_like(q, float("nan"))
        rc, err = _static_call(lib, pool, w, layer, q, out)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        diff = float((out - ref).abs().max())
        assert diff <= BF16_ATOL, diff
        assert torch.isfinite(out).all()


def test_static_entry_rejects_oversize_before_launch():
    import torch

    from pagellm_b200 import _lib

    lib = _lib.load()
    w, pool = _setup(12, 4)
    q = torch.zeros((600, w.H, w.D), device="cuda")
    out = torch.zeros_like(q)
    indptr = np.zeros(601, np.int64)
    ids = np.zeros(1, np.int32)
    ctx = np.ones(600, np.int64)
    rc = lib.pk_decode_attend_static(
        pool.handle, 0, w.H, 600, indptr.ctypes.data_as(C.POINTER(C.c_int64)),
        ids.ctypes.data_as(C.POINTER(C.c_int32)), ctx.ctypes.data_as(C.POINTER(C.c_int64)),
        q.data_ptr(), out.data_ptr(), None, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.PK_ERR_INVALID_ARG
    assert "static scratch" in _lib.last_error()
    # a plan larger than the 16 MiB array: 512 one-block sequences still need
    # (512 + CTAs) x 8 heads x 16 columns x 128 dims of float partials (> 40 MB)
    from pagellm_b200.cache import PagedKVPool

    class Shape:
        n_layers, n_kv_heads, head_dim = 1, 8, 128

    bp = PagedKVPool(Shape, 512, 16, "bfloat16")
    indptr = np.arange(513, dtype=np.int64)
    ids = np.arange(512, dtype=np.int32)
    ctx = np.full(512, 16, np.int64)
    qb = torch.zeros((512, 32, 128), device="cuda")
    ob = torch.zeros_like(qb)
    rc = lib.pk_decode_attend_static(
        bp.handle, 0, 32, 512, indptr.ctypes.data_as(C.POINTER(C.c_int64)),
        ids.ctypes.data_as(C.POINTER(C.c_int32)), ctx.ctypes.data_as(C.POINTER(C.c_int64)),
        qb.data_ptr(), ob.data_ptr(), None, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.PK_ERR_INVALID_ARG
    assert "scratch" in _lib.last_error()
    torch.cuda.synchronize()
    assert float(ob.abs().max()) == 0.0  # nothing was launched
