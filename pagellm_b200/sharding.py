"""Multi-GPU layouts of the paged KV cache (one process per GPU).

* Sequence-sharded (the default): every rank owns whole sequences - its own block pool,
  block tables and ``PagedBatch`` - so the hot path has no collective at all. Sequences are
  dealt longest first to the rank with the least total context (``shard_sequences``).
* Head-sharded (long contexts): every rank owns ``KVH / world`` KV heads (and their
  ``g`` query heads each) for every sequence; after attention the per-rank slices
  ``[rows, H/world, D]`` are all-gathered and interleaved back to ``[rows, H, D]``
  (``gather_heads``). Works over NCCL (CUDA tensors) and gloo (CPU tensors).

pagellm itself is single-process; these layouts are the multi-GPU form of its
``PagedBatch.write_and_attend`` (cache/paged.py:441-464), whose output they reproduce.
"""

from __future__ import annotations

from dataclasses import dataclass


def shard_sequences(lengths, world: int) -> list[list[int]]:
    """Sequence indices per rank: longest first, each to the rank with the smallest total
    context so far (ties to the lower rank); every rank's list is returned sorted."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    load = [0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        parts[r].append(i)
        load[r] += int(lengths[i])
    return [sorted(p) for p in parts]


@dataclass(frozen=True)
class HeadSlice:
    """The KV heads [kv0, kv1) and query heads [q0, q1) one rank owns."""

    kv0: int
    kv1: int
    q0: int
    q1: int


def head_slice(rank: int, world: int, n_kv_heads: int, n_heads: int) -> HeadSlice:
    if n_kv_heads % world:
        raise ValueError(f"{n_kv_heads} KV heads do not split over {world} ranks")
    if n_heads % n_kv_heads:
        raise ValueError("n_heads must be a multiple of n_kv_heads")
    per = n_kv_heads // world
    g = n_heads // n_kv_heads
    return HeadSlice(rank * per, (rank + 1) * per, rank * per * g, (rank + 1) * per * g)


def gather_heads(out_slice, group=None):
    """All-gather each rank's ``[rows, H/world, D]`` attention slice into ``[rows, H, D]``
    (rank r's slice lands at query heads [r*H/world, (r+1)*H/world))."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rows, hs, d = out_slice.shape
    buf = torch.empty((world * rows, hs, d), dtype=out_slice.dtype, device=out_slice.device)
    dist.all_gather_into_tensor(buf, out_slice.contiguous(), group=group)
    return buf.view(world, rows, hs, d).permute(1, 0, 2, 3).reshape(rows, world * hs, d)
