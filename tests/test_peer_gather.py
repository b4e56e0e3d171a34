"""The head-sharded output exchange over peer memory (pk_peer_gather_*), on 2 GPUs.

Each rank (a child process per GPU, NCCL for the handle exchange, 127.0.0.1 rendezvous)
owns KV heads [r*KVH/N, (r+1)*KVH/N) in the head-sharded layout; after its attention it
holds the slice [rows, H/N, D] of the step's output. One libpagekv launch stores every
slice into every rank's [rows, H, D] result and completes once all have landed. Checked:
the result equals the slices interleaved by head (bit for bit) on consecutive steps (both of
the alternating buffers), equals the NCCL all-gather path, and a rank that skips a step
makes the other rank's bounded wait report a timeout on the host, after which the GPU still
runs work. Skipped with fewer than 2 GPUs. NVLS is off (plain peer stores only).
"""

from __future__ import annotations

import os
import socket

import pytest

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, mode: str):
    import torch
    import torch.distributed as dist

    from pagellm_b200 import _lib
    from pagellm_b200.sharding import HeadGather, PeerHeadGather

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta

    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        rows, hs, d = 37, 8, 128
        pg = PeerHeadGather()
        if mode == "gather":
            ng = HeadGather()
            for step in range(5):
                # the slice a rank would hold: values that encode (step, rank, row, head, dim)
                g = torch.Generator(device=dev).manual_seed(1000 * step + rank)
                mine = torch.randn((rows, hs, d), generator=g, device=dev)
                full = pg(mine)
                pg.check()
                every = [torch.randn((rows, hs, d), generator=torch.Generator(device=dev).manual_seed(1000 * step + r),
                                     device=dev) for r in range(world)]
                want = torch.cat(every, dim=1)
                assert torch.equal(full, want), (rank, step)
                assert torch.equal(ng(mine), want), (rank, step)
        elif mode == "fused":
            _fused_steps(rank, world, dev, pg)
        else:
            g = torch.Generator(device=dev).manual_seed(rank)
            mine = torch.randn((rows, hs, d), generator=g, device=dev)
            pg(mine)
            pg.check()
            dist.barrier()
            if rank == 0:
                pg(mine)  # rank 1 skips this step: no slice and no flag from it
                with pytest.raises(_lib.DeviceTimeout):
                    pg.check()
                x = torch.ones(1024, device=dev)
                assert float((x * 2).sum()) == 2048.0  # the context still runs work
            dist.barrier()
        torch.cuda.synchronize()
        pg.close()
    finally:
        dist.destroy_process_group()


def _fused_steps(rank, world, dev, pg):
    """Head-sharded steps of a 2-layer bf16 pool (8 KV heads, g = 4, head_dim 128) split over
    the ranks: the fused launch (exchange inside the attention kernel) against the attention
    into a slice followed by the separate push, bit for bit, on consecutive steps; then a step
    with a 96-token chunk (wide-tile kernel), which takes the slice-and-push fallback."""
    import numpy as np
    import torch

    from pagellm_b200.cache import PagedBatch, PagedKVPool
    from pagellm_b200.sharding import head_slice

    KVH, H, D, bs = 8, 32, 128, 16
    sl = head_slice(rank, world, KVH, H)
    kvh, hs = sl.kv1 - sl.kv0, sl.q1 - sl.q0

    class Shape:
        n_layers, n_kv_heads, head_dim = 2, kvh, D

    rng = np.random.default_rng(7)  # same tables and lengths on every rank
    lens = rng.integers(200, 3000, size=24)
    nblk = [-(-int(L) // bs) + 8 for L in lens]
    nb = sum(nblk) + 16
    perm = rng.permutation(nb).astype(np.int32)
    tables, used = [], 0
    for n in nblk:
        tables.append(perm[used:used + n])
        used += n
    pool = PagedKVPool(Shape, nb, bs, "bfloat16")
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    for t in (pool.k, pool.v):
        t.copy_(torch.randn(t.shape, generator=g, device=dev).to(t.dtype))

    def step(starts, n_new, layer, seed, expect_fused):
        batch = PagedBatch(pool, tables, starts, n_new)
        rows = int(sum(n_new))
        gq = torch.Generator(device=dev).manual_seed(seed * 10 + rank)
        q = torch.randn((rows, hs, D), generator=gq, device=dev)
        k = torch.randn((rows, kvh, D), generator=gq, device=dev)
        v = torch.randn((rows, kvh, D), generator=gq, device=dev)
        fused = pg.write_and_attend(batch, layer, q, k, v, fused=True).clone()
        pg.check()
        slice_ = batch.write_and_attend(layer, q, k, v)  # the same rows appended again: same pool
        sep = pg(slice_).clone()
        pg.check()
        assert torch.equal(fused, sep), (rank, seed)
        dflt = pg.write_and_attend(batch, layer, q, k, v, fused=False).clone()  # attention + push launch
        pg.check()
        assert torch.equal(dflt, sep), (rank, seed)
        assert torch.equal(fused[:, sl.q0:sl.q1], slice_), (rank, seed)
        assert torch.isfinite(fused).all()
        st = batch.stats()
        assert (st["wide_items"] == 0) == expect_fused, st

    starts = [int(L) for L in lens]
    for i in range(3):  # decode steps on alternating result buffers and layers
        step([s + i for s in starts], [1] * len(lens), i % 2, i, True)
    n_new = [1] * len(lens)
    n_new[0] = 96  # a prefill chunk: wide-tile kernel, slice + push
    step([s + 3 for s in starts], n_new, 0, 9, False)


def _run(mode: str):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.spawn(_worker, args=(2, _free_port(), mode), nprocs=2, join=True)


def test_peer_gather_matches_interleave_and_nccl():
    _run("gather")


def test_peer_gather_missing_peer_times_out_on_host():
    _run("timeout")


def test_fused_exchange_matches_attention_then_push():
    _run("fused")
