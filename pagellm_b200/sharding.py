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


class HeadGather:
    """All-gather of each rank's ``[rows, H/world, D]`` attention slice into ``[rows, H, D]``
    (rank r's slice lands at query heads [r*H/world, (r+1)*H/world)), with reusable buffers.

    CUDA tensors: ``all_gather_into_tensor`` (NCCL) into ``[world, rows, H/world, D]``, then
    libpagekv's interleave kernel writes the ``[rows, H, D]`` result. CPU tensors (gloo, the
    multi-process tests) interleave with a tensor permute."""

    def __init__(self, group=None):
        self.group = group
        self._buf = None
        self._out = None

    def __call__(self, out_slice):
        import torch
        import torch.distributed as dist

        world = dist.get_world_size(self.group)
        rows, hs, d = out_slice.shape
        shape = (world * rows, hs, d)
        if self._buf is None or self._buf.shape != shape or self._buf.device != out_slice.device \
                or self._buf.dtype != out_slice.dtype:
            self._buf = torch.empty(shape, dtype=out_slice.dtype, device=out_slice.device)
            self._out = torch.empty((rows, world * hs, d), dtype=out_slice.dtype, device=out_slice.device)
        dist.all_gather_into_tensor(self._buf, out_slice.contiguous(), group=self.group)
        if not out_slice.is_cuda:
            return self._buf.view(world, rows, hs, d).permute(1, 0, 2, 3).reshape(rows, world * hs, d)
        if out_slice.dtype != torch.float32:
            raise ValueError("head gather on the GPU takes float32 slices")
        from . import _lib

        st = torch.cuda.current_stream(out_slice.device).cuda_stream
        _lib.check(_lib.load().pk_gather_interleave(self._buf.data_ptr(), self._out.data_ptr(), world, rows,
                                                    hs * d, st))
        return self._out


class PeerHeadGather:
    """The head-sharded all-gather as one libpagekv launch per step over peer memory: every
    rank stores its ``[rows, H/world, D]`` float32 slice straight into every rank's
    ``[rows, H, D]`` result buffer (IPC-mapped over NVLink) and the launch completes once all
    slices have landed. Buffers are created on the first call (a collective: every rank calls
    with the same shape) and grown collectively when a larger result is needed. The returned
    tensor is the library's buffer: it stays valid until the call after next."""

    def __init__(self, group=None):
        self.group = group
        self._g = None
        self._bytes = 0

    def _setup(self, nbytes: int, device):
        import ctypes as C

        import torch.distributed as dist

        from . import _lib

        lib = _lib.load()
        self.close()
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        h = C.c_void_p()
        _lib.check(lib.pk_peer_gather_create(device.index, world, rank, nbytes, C.byref(h)))
        self._g = h.value
        self._bytes = nbytes
        mine = C.create_string_buffer(64)
        _lib.check(lib.pk_peer_gather_handle(self._g, mine))
        every = [None] * world
        dist.all_gather_object(every, mine.raw, group=self.group)
        _lib.check(lib.pk_peer_gather_open(self._g, b"".join(every)))

    def __call__(self, out_slice):
        import ctypes as C

        import torch
        import torch.distributed as dist

        from . import _lib

        if not out_slice.is_cuda or out_slice.dtype != torch.float32:
            raise ValueError("peer head gather takes float32 CUDA slices")
        world = dist.get_world_size(self.group)
        rows, hs, d = out_slice.shape
        nbytes = max(16, rows * world * hs * d * 4)
        if self._g is None or nbytes > self._bytes:
            self._setup(nbytes, out_slice.device)
        src = out_slice if out_slice.is_contiguous() and out_slice.data_ptr() % 16 == 0 else out_slice.contiguous()
        res = C.c_void_p()
        st = torch.cuda.current_stream(out_slice.device).cuda_stream
        _lib.check(_lib.load().pk_peer_gather_heads(self._g, src.data_ptr(), rows, hs * d, C.byref(res), st))
        from .cache.paged import _CudaArray

        return torch.as_tensor(_CudaArray(res.value, (rows, world * hs, d), "<f4", self), device=out_slice.device)

    def write_and_attend(self, batch, layer: int, q, k, v, fused=None):
        """The head-sharded step: ``batch.write_and_attend(layer, q, k, v)`` over this rank's
        heads (``q`` [rows, H/world, D], ``k``/``v`` [rows, KVH/world, D], float32 CUDA
        tensors) and the exchange of the output slices. ``fused=True``: one launch, the
        attention kernel stores every output row into every rank's result and exchanges the
        flags at its end; ``fused=False``: the attention, then one push launch. ``None`` picks
        by world size from B200 measurements of C5's head-sharded step: fused at 2 ranks
        (439.5 against 444.9 us), push beyond (8 ranks: 145.4 against 159.0 us, since only the
        few merging warps issue the fused kernel's tail stores to 8 ranks). Returns the
        [rows, H, D] result (the library's buffer, valid until the call after next).
        Collective: every rank calls it for the same step, with the same rows."""
        import ctypes as C

        import torch
        import torch.distributed as dist

        from . import _lib

        for t in (q, k, v):
            if not t.is_cuda or t.dtype != torch.float32:
                raise ValueError("write_and_attend takes float32 CUDA tensors")
        world = dist.get_world_size(self.group)
        if fused is None:
            fused = world <= 2
        if not fused:
            return self(batch.write_and_attend(layer, q, k, v))
        rows, hs, d = q.shape
        nbytes = max(16, rows * world * hs * d * 4)
        if self._g is None or nbytes > self._bytes:
            self._setup(nbytes, q.device)
        q, k, v = (t if t.is_contiguous() else t.contiguous() for t in (q, k, v))
        res = C.c_void_p()
        st = torch.cuda.current_stream(q.device).cuda_stream
        _lib.check(_lib.load().pk_peer_gather_write_and_attend(self._g, batch._b, layer, hs, q.data_ptr(),
                                                               k.data_ptr(), v.data_ptr(), C.byref(res), st))
        from .cache.paged import _CudaArray

        return torch.as_tensor(_CudaArray(res.value, (rows, world * hs, d), "<f4", self), device=q.device)

    def check(self, stream=None) -> None:
        """Synchronise and raise DeviceTimeout if a peer's slice did not arrive in time."""
        import torch

        from . import _lib

        if self._g is not None:
            st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
            _lib.check(_lib.load().pk_peer_gather_check(self._g, st))

    def close(self) -> None:
        """Collective (every rank calls it): waits until no rank's launch can still be storing
        into this rank's buffers, then unmaps the peers' and frees this rank's."""
        if self._g is not None:
            import torch
            import torch.distributed as dist

            from . import _lib

            torch.cuda.synchronize()
            if dist.is_initialized():
                dist.barrier(group=self.group)
            _lib.load().pk_peer_gather_destroy(self._g)
            self._g = None

    def __del__(self):
        # not collective: only frees what a missed close() left behind
        if self._g is not None:
            try:
                from . import _lib

                _lib.load().pk_peer_gather_destroy(self._g)
            except Exception:
                pass
            self._g = None


def gather_heads(out_slice, group=None):
    """One-off :class:`HeadGather` call (fresh buffers; the returned tensor is the caller's)."""
    return HeadGather(group)(out_slice)
