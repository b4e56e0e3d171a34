"""Device-resident drop-in for pagellm's paged KV cache (pagellm src/pagellm/cache/paged.py).

Same names, arguments and errors as pagellm:

* ``PagedKVPool(cfg, num_blocks, block_size, dtype)`` (paged.py:282-300) - K/V live on the
  GPU in a pool owned by libpagekv; ``.k/.v/.k_flat/.v_flat`` are torch views of it.
* ``PagedBatch(pool, block_tables, starts, n_new, attn, batch_decode)`` (paged.py:383-464)
  with ``.positions``, ``.slots``, ``.offsets`` and ``write_and_attend(layer, q, k, v)``.
* ``slot_mapping``, ``paged_attention``, ``batched_decode_attention`` (paged.py:303-380).
* ``BlockAllocator``, ``BlockManager``, ``BlockTable``, ``OutOfBlocks``, ``block_hash``
  (paged.py:38-274): bookkeeping on the host, free list / ref counts / LRU in C++.

Every computation runs in libpagekv's CUDA kernels; there is no CPU path. ``attn`` accepts
pagellm's ``"gather"`` and ``"paged"`` (both run the same kernels: the device kernel reads
the pool block by block through the table, which is what both of pagellm's modes compute).
"""

from __future__ import annotations

import ctypes as C
import itertools
import sys

import numpy as np

from .. import _lib
from .block_manager import BlockAllocator, BlockManager, BlockTable, OutOfBlocks, block_hash

__all__ = [
    "BlockAllocator",
    "BlockManager",
    "BlockTable",
    "OutOfBlocks",
    "PagedBatch",
    "PagedKVPool",
    "batched_decode_attention",
    "block_hash",
    "paged_attention",
    "slot_mapping",
]


def _torch():
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("pagellm_b200 needs a CUDA device (B200, sm_100a); none is visible")
    return torch


def _stream(device) -> int:
    """Raw handle of the caller's current torch stream on ``device``."""
    torch = _torch()
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None and device.index is not None and torch.cuda.is_initialized():
        return raw(device.index)  # no Stream object: this runs on every step
    return torch.cuda.current_stream(device).cuda_stream


def _addr(a: np.ndarray) -> int:
    """Address of a C-contiguous array's data; the buffer-protocol route is several times
    cheaper than ``ndarray.ctypes`` and is taken for every writable, non-empty array."""
    try:
        return C.addressof(C.c_char.from_buffer(a))
    except (TypeError, ValueError):  # read-only or empty
        return a.ctypes.data


def _dtype_code(dtype):
    """(libpagekv code, canonical name) for numpy / torch / string dtypes."""
    name = getattr(dtype, "name", None) or str(dtype)
    name = name.replace("torch.", "").lower()
    if name in ("float32", "f32", "fp32", "<f4", "float"):
        return _lib.PK_F32, "float32"
    if name in ("bfloat16", "bf16"):
        return _lib.PK_BF16, "bfloat16"
    try:
        if np.dtype(dtype) == np.float32:
            return _lib.PK_F32, "float32"
    except TypeError:
        pass
    raise ValueError(f"unsupported KV pool dtype {dtype!r} (float32 or bfloat16)")


class _CudaArray:
    """Zero-copy __cuda_array_interface__ view of library-owned device memory; holds a
    reference to the owner so the memory outlives every tensor made from it."""

    def __init__(self, addr: int, shape, typestr: str, owner):
        self.__cuda_array_interface__ = {
            "shape": tuple(int(s) for s in shape),
            "typestr": typestr,
            "data": (int(addr), False),
            "version": 3,
            "strides": None,
        }
        self._owner = owner


class _Handle:
    def __init__(self, ptr: int, destroy, device_index: int):
        self.ptr = ptr
        self._destroy = destroy
        self._device = device_index

    def close(self):
        if self.ptr:
            self._destroy(self.ptr)
            self.ptr = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PagedKVPool:
    """Physical KV storage ``(layers, num_blocks, block_size, kv_heads, head_dim)`` on a GPU.

    ``cfg`` is anything with ``n_layers``, ``n_kv_heads`` and ``head_dim`` (pagellm's
    ``ModelConfig`` works). ``dtype``: float32 (pagellm's default) or bfloat16. The pool is
    zero-filled like pagellm's ``np.zeros`` pool (paged.py:287-289).
    """

    def __init__(self, cfg, num_blocks: int, block_size: int, dtype=np.float32, device=None):
        torch = _torch()
        lib = _lib.load()
        self.block_size = int(block_size)
        self.num_blocks = int(num_blocks)
        self.n_layers = int(cfg.n_layers)
        self.n_kv_heads = int(cfg.n_kv_heads)
        self.head_dim = int(cfg.head_dim)
        code, self.dtype_name = _dtype_code(dtype)
        self._code = code
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None
                                   else torch.device(device).index or 0)
        h = C.c_void_p()
        _lib.check(lib.pk_pool_create(self.n_layers, self.num_blocks, self.block_size,
                                      self.n_kv_heads, self.head_dim, code, self.device.index,
                                      C.byref(h)))
        self._h = _Handle(h.value, lib.pk_pool_destroy, self.device.index)
        kp, vp, nbytes = C.c_void_p(), C.c_void_p(), C.c_int64()
        _lib.check(lib.pk_pool_buffers(self._h.ptr, C.byref(kp), C.byref(vp), C.byref(nbytes)))
        self._nbytes = nbytes.value
        shape = (self.n_layers, self.num_blocks, self.block_size, self.n_kv_heads, self.head_dim)
        typestr = "<f4" if code == _lib.PK_F32 else "<i2"

        def view(addr):
            t = torch.as_tensor(_CudaArray(addr, shape, typestr, self._h), device=self.device)
            return t if code == _lib.PK_F32 else t.view(torch.bfloat16)

        self.k = view(kp.value)
        self.v = view(vp.value)
        flat = (self.n_layers, self.num_blocks * self.block_size, self.n_kv_heads, self.head_dim)
        self.k_flat = self.k.view(flat)
        self.v_flat = self.v.view(flat)
        self._idle_batches: list[int] = []
        self._batch_prefix_mode: dict[int, int] = {}  # handle -> prefix-sharing mode it holds

    # ------------------------------------------------------------------ pagellm API
    def copy_block(self, src: int, dst: int) -> None:
        """k[:, dst] = k[:, src]; v[:, dst] = v[:, src] (paged.py:294-296)."""
        self.copy_blocks([(src, dst)])

    def copy_blocks(self, pairs) -> None:
        """All copy-on-write pairs of a step in one launch, in list order semantics."""
        arr = np.ascontiguousarray(np.asarray(pairs, dtype=np.int64).reshape(-1, 2))
        if len(arr) == 0:
            return
        lib = _lib.load()
        _lib.check(lib.pk_pool_copy_blocks(self._h.ptr, arr.ctypes.data_as(C.POINTER(C.c_int64)),
                                           len(arr), _stream(self.device)))

    @property
    def nbytes(self) -> int:
        return self._nbytes

    # ------------------------------------------------------------------ extras
    @property
    def tensor_core_path(self) -> tuple[bool, str]:
        """(enabled, reason) for the tensor-core attention kernel on this pool."""
        en, ph, st, why = C.c_int(), C.c_int(), C.c_int(), C.c_char_p()
        _lib.check(_lib.load().pk_pool_tc_info(self._h.ptr, C.byref(en), C.byref(ph), C.byref(st),
                                               C.byref(why)))
        return bool(en.value), (why.value or b"").decode()

    @property
    def handle(self) -> int:
        return self._h.ptr

    def _acquire_batch(self) -> int:
        if self._idle_batches:
            return self._idle_batches.pop()
        h = C.c_void_p()
        _lib.check(_lib.load().pk_batch_create(self._h.ptr, C.byref(h)))
        return h.value

    def _release_batch(self, h: int) -> None:
        self._idle_batches.append(h)

    def close(self) -> None:
        lib = _lib.load()
        for h in self._idle_batches:
            lib.pk_batch_destroy(h)
        self._idle_batches.clear()
        self._h.close()

    def __del__(self):
        try:
            lib = _lib.load()
            for h in self._idle_batches:
                lib.pk_batch_destroy(h)
            self._idle_batches.clear()
        except Exception:
            pass


class _PinnedResults:
    """Page-locked float32 result buffers, reused once the caller has dropped them.

    Device-to-host copies into pageable memory run at a fraction of DMA speed, and pinning
    a fresh buffer per call costs more than the copy; so results are handed out in pinned
    arrays from a small cache, and a cached array is reused only when nothing outside the
    cache still refers to it."""

    def __init__(self, keep: int = 4):
        self.keep = keep
        self.bufs: list[np.ndarray] = []

    def get(self, shape) -> np.ndarray:
        shape = tuple(int(x) for x in shape)
        for b in self.bufs:
            # references: the list slot, the loop variable, getrefcount's argument
            if b.shape == shape and sys.getrefcount(b) <= 3:
                return b
        torch = _torch()
        b = torch.empty(shape, dtype=torch.float32, pin_memory=True).numpy()
        self.bufs.append(b)
        if len(self.bufs) > self.keep:
            self.bufs.pop(0)
        return b


_PINNED = _PinnedResults()


def _pinned_empty(shape) -> np.ndarray:
    return _PINNED.get(shape)


def _aligned(t):
    """``t`` itself when its data starts on a 16-byte boundary, else an aligned copy."""
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _csr(block_tables):
    """(indptr int64, ids int32) from a list of per-sequence block lists / arrays."""
    if isinstance(block_tables, tuple) and len(block_tables) == 2 and isinstance(block_tables[0], np.ndarray) \
            and block_tables[0].ndim == 1 and len(block_tables[0]) and block_tables[0][0] == 0 \
            and block_tables[1].dtype == np.int32:
        return np.ascontiguousarray(block_tables[0], np.int64), np.ascontiguousarray(block_tables[1])
    lens = np.fromiter((len(t) for t in block_tables), dtype=np.int64, count=len(block_tables))
    indptr = np.zeros(len(lens) + 1, dtype=np.int64)
    np.cumsum(lens, out=indptr[1:])
    total = int(indptr[-1])
    if total and all(isinstance(t, np.ndarray) for t in block_tables):
        ids = np.concatenate(block_tables).astype(np.int32, copy=False)
    else:
        flat = np.fromiter(itertools.chain.from_iterable(block_tables), dtype=np.int64, count=total)
        if total and (flat.min() < -(2 ** 31) or flat.max() >= 2 ** 31):
            raise IndexError("block id outside the int32 range")
        ids = flat.astype(np.int32)
    return indptr, np.ascontiguousarray(ids)


class PagedBatch:
    """KVBackend for a batch of sequences whose K/V live in a device ``PagedKVPool``.

    Mirrors pagellm's ``PagedBatch`` (paged.py:383-464). The constructor validates and uploads
    the block tables once per step and computes the slot mapping on the device;
    ``write_and_attend`` is one layer: append the new K/V at their slots, then causal GQA
    attention of every row over its sequence's cache.

    ``block_tables`` may also be given as a CSR pair ``(indptr int64, ids int32)``.
    ``q, k, v`` may be numpy arrays (result returned as numpy, dtype of ``q``) or float32
    CUDA tensors on the pool's device (result returned as a CUDA tensor, no host copies).
    """

    def __init__(self, pool: PagedKVPool, block_tables, starts, n_new, attn: str = "gather",
                 batch_decode: bool = True):
        if attn not in ("gather", "paged"):
            raise ValueError(attn)
        self.pool, self.attn, self.batch_decode = pool, attn, batch_decode
        self.block_tables, self.starts, self.n_new = block_tables, starts, n_new
        starts_a = np.ascontiguousarray(np.asarray(starts, dtype=np.int64).reshape(-1))
        n_new_a = np.ascontiguousarray(np.asarray(n_new, dtype=np.int64).reshape(-1))
        if len(starts_a) != len(n_new_a):
            raise ValueError("starts and n_new differ in length")
        indptr, ids = _csr(block_tables)
        if len(indptr) - 1 != len(n_new_a):
            raise ValueError("block_tables and n_new differ in length")
        self._starts_a, self._n_new_a = starts_a, n_new_a
        self._offsets = None
        self._positions = None
        lib = _lib.load()
        self._lib = lib
        self._b = pool._acquire_batch()
        if pool._batch_prefix_mode.get(self._b, 1) != 1:  # a recycled handle: back to the default
            _lib.check(lib.pk_batch_set_prefix_sharing(self._b, 1))
            pool._batch_prefix_mode[self._b] = 1
        self._prefix_sharing = "auto"
        rows = C.c_int64()
        _lib.check(lib.pk_batch_plan(self._b, len(n_new_a), _addr(indptr), _addr(ids), _addr(starts_a),
                                     _addr(n_new_a), C.byref(rows), _stream(pool.device)))
        self.num_rows = rows.value
        self._slots = None

    def __del__(self):
        # the handle goes back to the pool for the next step's batch
        b = getattr(self, "_b", None)
        if b is not None:
            try:
                self.pool._release_batch(b)
            except Exception:
                pass
            self._b = None

    # ------------------------------------------------------------------ step metadata
    @property
    def offsets(self) -> np.ndarray:
        """First row of every sequence in the flat batch (paged.py:410), plus the total."""
        if self._offsets is None:
            off = np.zeros(len(self._n_new_a) + 1, dtype=np.int64)
            np.cumsum(self._n_new_a, out=off[1:])
            self._offsets = off.astype(int)
        return self._offsets

    @property
    def positions(self) -> np.ndarray:
        """int64 absolute position of every new row (paged.py:412-414)."""
        if self._positions is None:
            total = int(self.offsets[-1])
            self._positions = (np.repeat(self._starts_a - self.offsets[:-1], self._n_new_a)
                               + np.arange(total, dtype=np.int64)) if total else np.zeros(0, np.int64)
        return self._positions

    @property
    def slots(self) -> np.ndarray:
        """int64 pool slot of every new row, as computed by the device slot-mapping kernel."""
        if self._slots is None:
            self._slots = self.slots_device().cpu().numpy()
        return self._slots

    def slots_device(self):
        torch = _torch()
        pos, sl = C.c_void_p(), C.c_void_p()
        _lib.check(self._lib.pk_batch_rows(self._b, C.byref(pos), C.byref(sl)))
        n = self.num_rows
        if n == 0:
            return torch.zeros(0, dtype=torch.int64, device=self.pool.device)
        return torch.as_tensor(_CudaArray(sl.value, (n,), "<i8", self), device=self.pool.device)

    def stats(self) -> dict:
        s = (C.c_int64 * 8)()
        _lib.check(self._lib.pk_batch_stats(self._b, s))
        keys = ("rows", "tc_units", "tc_ctas", "tc_blocks", "split_units", "generic_rows", "launches",
                "wide_items")
        return dict(zip(keys, list(s)))

    def io_stats(self) -> dict:
        """Bytes the last host-buffer ``write_and_attend`` moved: ``h2d``, ``d2h`` (a copy
        after the kernels) and ``direct`` (stored by the kernels into the page-locked result)."""
        s = (C.c_int64 * 3)()
        _lib.check(self._lib.pk_batch_io_stats(self._b, s))
        return dict(zip(("h2d", "d2h", "direct"), list(s)))

    _PREFIX_MODES = {False: 0, "off": 0, True: 1, "auto": 1, "always": 2}

    @property
    def prefix_sharing(self) -> str:
        """Shared-prefix (cascade) attention for sequences whose block tables begin with the
        same blocks: "auto" (default: where a cost estimate favours it), "always" or "off".
        Not in pagellm; results are the same either way within floating-point rounding."""
        return self._prefix_sharing

    @prefix_sharing.setter
    def prefix_sharing(self, mode) -> None:
        if mode not in self._PREFIX_MODES:
            raise ValueError(f"prefix_sharing must be 'off', 'auto' or 'always', not {mode!r}")
        code = self._PREFIX_MODES[mode]
        _lib.check(self._lib.pk_batch_set_prefix_sharing(self._b, code))
        self.pool._batch_prefix_mode[self._b] = code
        self._prefix_sharing = ("off", "auto", "always")[code]

    def prefix_stats(self) -> dict:
        s = (C.c_int64 * 4)()
        _lib.check(self._lib.pk_batch_prefix_stats(self._b, s))
        return dict(zip(("groups", "items", "shared_keys", "token_keys"), list(s)))

    # ------------------------------------------------------------------ per layer
    def write_and_attend(self, layer: int, q, k, v):
        return self._run(layer, q, k, v, append=True)

    def attend(self, layer: int, q):
        """Attention only: the read half of ``write_and_attend`` (no append)."""
        return self._run(layer, q, None, None, append=False)

    def _run(self, layer, q, k, v, append):
        P = self.pool
        if q.ndim != 3 or q.shape[0] != self.num_rows or q.shape[2] != P.head_dim:
            raise ValueError(f"q must be (rows={self.num_rows}, H, {P.head_dim}), got {tuple(q.shape)}")
        H = int(q.shape[1])
        if append:
            want = (self.num_rows, P.n_kv_heads, P.head_dim)
            if tuple(k.shape) != want or tuple(v.shape) != want:
                raise ValueError(f"k, v must be {want}")
        st = _stream(P.device)
        if hasattr(q, "is_cuda"):
            torch = _torch()
            qd = _aligned(q.to(P.device, torch.float32).contiguous())
            out = torch.empty_like(qd)
            if append:
                kd = _aligned(k.to(P.device, torch.float32).contiguous())
                vd = _aligned(v.to(P.device, torch.float32).contiguous())
                rc = self._lib.pk_batch_write_and_attend(self._b, layer, H, qd.data_ptr(),
                                                         kd.data_ptr(), vd.data_ptr(),
                                                         out.data_ptr(), st)
            else:
                rc = self._lib.pk_batch_attend(self._b, layer, H, qd.data_ptr(), out.data_ptr(), st)
            _lib.check(rc)
            return out if q.dtype == torch.float32 else out.to(q.dtype)
        qh = np.ascontiguousarray(q, dtype=np.float32)
        out = _pinned_empty(qh.shape)
        if append:
            kh = np.ascontiguousarray(k, dtype=np.float32)
            vh = np.ascontiguousarray(v, dtype=np.float32)
            _lib.check(self._lib.pk_batch_write_and_attend_host(
                self._b, layer, H, _addr(qh), _addr(kh), _addr(vh), _addr(out), st))
        else:
            torch = _torch()
            qd = torch.from_numpy(qh).to(P.device)
            od = torch.empty_like(qd)
            _lib.check(self._lib.pk_batch_attend(self._b, layer, H, qd.data_ptr(), od.data_ptr(), st))
            out = od.cpu().numpy()
        return out.astype(q.dtype, copy=False)

    def check(self) -> None:
        """Synchronise and raise ``DeviceTimeout`` if a bounded device wait gave up."""
        _lib.check(self._lib.pk_batch_check(self._b, _stream(self.pool.device)))


# ---------------------------------------------------------------------- free functions
def slot_mapping(block_table, positions, block_size: int) -> np.ndarray:
    """Physical slot for each logical position (paged.py:303-306), computed on the GPU.

    Host inputs give a numpy int64 result; CUDA tensors give a CUDA tensor."""
    torch = _torch()
    lib = _lib.load()
    on_dev = hasattr(positions, "is_cuda") and positions.is_cuda
    dev = positions.device if on_dev else torch.device("cuda", torch.cuda.current_device())
    tbl = torch.as_tensor(np.asarray(block_table, dtype=np.int64) if not hasattr(block_table, "is_cuda")
                          else block_table).to(dev, torch.int32).contiguous()
    pos = torch.as_tensor(positions if on_dev else np.asarray(positions, dtype=np.int64))
    pos = pos.to(dev, torch.int64).contiguous()
    out = torch.empty_like(pos)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(lib.pk_slot_mapping(tbl.data_ptr(), tbl.numel(), pos.data_ptr(), pos.numel(),
                                   int(block_size), out.data_ptr(), err.data_ptr(),
                                   torch.cuda.current_stream(dev).cuda_stream))
    if int(err.item()):
        raise IndexError("position outside the block table")
    return out if on_dev else out.cpu().numpy().reshape(np.shape(positions))


class _Shape:
    def __init__(self, n_layers, n_kv_heads, head_dim):
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim


def _pool_dtype_of(a):
    name = str(getattr(a, "dtype", "float32"))
    return "bfloat16" if "bfloat16" in name else np.float32


def paged_attention(q, k_pool, v_pool, block_table, context_len: int, q_start: int):
    """Causal attention read through a block table (paged.py:309-352), on the GPU.

    q: (n, H, d) at positions q_start..q_start+n-1; k_pool, v_pool: (num_blocks, bs, KVH, d)
    for one layer. The blocks are staged into a one-layer device pool; ``context_len`` must
    be ``q_start + n`` as in every pagellm call (paged.py:461-463)."""
    torch = _torch()
    n = int(q.shape[0])
    if int(context_len) != int(q_start) + n:
        raise ValueError("context_len must equal q_start + len(q)")
    nb, bs, kvh, d = (int(x) for x in k_pool.shape)
    pool = PagedKVPool(_Shape(1, kvh, d), nb, bs, _pool_dtype_of(k_pool))
    pool.k[0].copy_(torch.as_tensor(np.asarray(k_pool, np.float32) if not hasattr(k_pool, "is_cuda")
                                    else k_pool).to(pool.k.dtype))
    pool.v[0].copy_(torch.as_tensor(np.asarray(v_pool, np.float32) if not hasattr(v_pool, "is_cuda")
                                    else v_pool).to(pool.v.dtype))
    batch = PagedBatch(pool, [list(block_table)], [int(q_start)], [n], attn="paged")
    return batch.attend(0, q)


def batched_decode_attention(q, k_ctx, v_ctx, valid):
    """One query per sequence over padded contexts (paged.py:355-380), on the GPU.

    Each sequence's valid keys are packed into a device pool and attended as a decode row;
    what the padding holds never reaches the kernel. A row with no valid key is NaN, as in
    the numpy original."""
    S, H, d = (int(x) for x in q.shape)
    k_ctx = np.asarray(k_ctx, dtype=np.float32)
    v_ctx = np.asarray(v_ctx, dtype=np.float32)
    valid = np.asarray(valid, dtype=bool)
    kvh = int(k_ctx.shape[2])
    lens = valid.sum(axis=1)
    live = np.nonzero(lens > 0)[0]
    out = np.full(q.shape, np.nan, dtype=np.asarray(q).dtype)
    if len(live) == 0:
        return out
    bs = 16
    nblk = [-(-int(lens[i]) // bs) for i in live]
    pool = PagedKVPool(_Shape(1, kvh, d), max(1, sum(nblk)), bs, np.float32)
    kf = np.zeros((sum(nblk) * bs, kvh, d), np.float32)
    vf = np.zeros_like(kf)
    tables, base = [], 0
    for i, nb in zip(live, nblk):
        kf[base * bs: base * bs + lens[i]] = k_ctx[i][valid[i]]
        vf[base * bs: base * bs + lens[i]] = v_ctx[i][valid[i]]
        tables.append(list(range(base, base + nb)))
        base += nb
    torch = _torch()
    pool.k_flat[0].copy_(torch.from_numpy(kf))
    pool.v_flat[0].copy_(torch.from_numpy(vf))
    batch = PagedBatch(pool, tables, [int(lens[i]) - 1 for i in live], [1] * len(live))
    out[live] = batch.attend(0, np.asarray(q)[live])
    return out
