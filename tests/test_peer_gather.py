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
