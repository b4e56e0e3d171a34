"""Multi-process (world size 2, gloo, CPU) checks of the multi-GPU layouts: sequence
sharding and head sharding reproduce the single-process result. Compute is the CPU oracle;
what is tested is the partitioning, the head all-gather and the reassembly."""

from __future__ import annotations

import os
import socket
import tempfile

import numpy as np
import pytest
import torch.multiprocessing as mp

from pagellm_b200.sharding import head_slice, shard_sequences


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(seed=0, nseq=5, H=16, KVH=4, D=32, bs=16):
    from oracle import paged_oracle as po

    rng = np.random.default_rng(seed)
    L = rng.integers(5, 90, nseq)
    nb = int(sum(-(-int(x) // bs) for x in L)) + 3
    perm = rng.permutation(nb)
    tables, used = [], 0
    for x in L:
        n = -(-int(x) // bs)
        tables.append(perm[used:used + n].tolist())
        used += n
    kp = rng.standard_normal((nb * bs, KVH, D)).astype(np.float32)
    vp = rng.standard_normal((nb * bs, KVH, D)).astype(np.float32)
    q = rng.standard_normal((nseq, H, D)).astype(np.float32)
    starts = (L - 1).tolist()
    meta = po.StepMeta(tables, starts, [1] * nseq, bs)
    return L, tables, kp, vp, q, meta


def _full(L, tables, kp, vp, q, meta):
    from oracle import paged_oracle as po

    out = np.empty_like(q)
    for i in range(len(L)):
        cs = meta.ctx_slots[i]
        out[i:i + 1] = po.attention_dense(q[i:i + 1], kp[cs], vp[cs], int(L[i]) - 1)
    return out


def _worker(rank, world, port, path, mode):
    import torch
    import torch.distributed as dist

    from oracle import paged_oracle as po
    from pagellm_b200.sharding import gather_heads

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    L, tables, kp, vp, q, meta = _problem()
    H, KVH = q.shape[1], kp.shape[1]
    if mode == "head":
        hs = head_slice(rank, world, KVH, H)
        mine = np.empty((len(L), hs.q1 - hs.q0, q.shape[2]), np.float32)
        for i in range(len(L)):
            cs = meta.ctx_slots[i]
            mine[i:i + 1] = po.attention_dense(q[i:i + 1, hs.q0:hs.q1], kp[cs, hs.kv0:hs.kv1],
                                               vp[cs, hs.kv0:hs.kv1], int(L[i]) - 1)
        full = gather_heads(torch.from_numpy(mine)).numpy()
    else:
        parts = shard_sequences(L, world)
        mine = {i: po.attention_dense(q[i:i + 1], kp[meta.ctx_slots[i]], vp[meta.ctx_slots[i]],
                                      int(L[i]) - 1) for i in parts[rank]}
        got = [None] * world
        dist.all_gather_object(got, mine)
        full = np.empty_like(q)
        for d in got:
            for i, o in d.items():
                full[i:i + 1] = o
    if rank == 0:
        np.save(path, full)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["head", "seq"])
def test_two_rank_layout_reproduces_single_process(mode):
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "out.npy")
        mp.start_processes(_worker, args=(2, _port(), path, mode), nprocs=2, join=True,
                           start_method="spawn")
        got = np.load(path)
    ref = _full(*_problem())
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6)


def test_shard_sequences_longest_first_balance():
    L = [100, 7, 300, 250, 250, 9, 40, 41]
    parts = shard_sequences(L, 3)
    assert sorted(i for p in parts for i in p) == list(range(len(L)))
    loads = [sum(L[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= max(L)
    assert parts[0][0] == 2 or 2 in parts[0]  # the longest goes to rank 0 first
    assert shard_sequences([5, 5], 1) == [[0, 1]]
    with pytest.raises(ValueError):
        shard_sequences([1], 0)


def test_head_slice_partition():
    sl = [head_slice(r, 4, 8, 64) for r in range(4)]
    assert [(s.kv0, s.kv1) for s in sl] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert [(s.q0, s.q1) for s in sl] == [(0, 16), (16, 32), (32, 48), (48, 64)]
    with pytest.raises(ValueError):
        head_slice(0, 3, 8, 64)


def _dying_worker(rank, world, port, path):
    """Rank 1 leaves after joining the group (between steps, nothing in flight); rank 0
    must learn of it from its next collective, through the process group's short timeout,
    as an exception on the host - no device is involved."""
    import time
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from pagellm_b200.sharding import gather_heads

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    dist.barrier()  # both ranks reached the step boundary
    if rank == 1:
        return  # the rank dies here: its process exits without the next collective
    t0 = time.time()
    try:
        gather_heads(torch.zeros((4, 2, 8)))
        outcome = "no error"
    except Exception as e:  # noqa: BLE001 - gloo raises RuntimeError subclasses
        outcome = f"detected after {time.time() - t0:.1f} s: {type(e).__name__}"
    with open(path, "w") as f:
        f.write(outcome)


def test_dead_rank_is_detected_on_the_host():
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "outcome.txt")
        mp.start_processes(_dying_worker, args=(2, _port(), path), nprocs=2, join=True,
                           start_method="spawn")
        outcome = open(path).read()
    assert outcome.startswith("detected"), outcome
    assert float(outcome.split()[2]) < 30.0, outcome
