"""ctypes binding of libpagekv.so (the C ABI declared in include/pagekv.h).

The library is built in-tree by ``pagellm_b200.build``. Loading fails loudly if it is
missing: there is no CPU fallback for anything in this package.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libpagekv.so"

PK_OK = 0
PK_ERR_INVALID_ARG = 1
PK_ERR_OUT_OF_RANGE = 2
PK_ERR_CUDA = 3
PK_ERR_OUT_OF_BLOCKS = 4
PK_ERR_DOUBLE_FREE = 5
PK_ERR_TIMEOUT = 6
PK_ERR_DUPLICATE = 7
PK_ERR_NOT_FOUND = 8
PK_ERR_UNSUPPORTED = 9

PK_F32 = 0
PK_BF16 = 1

_p = C.c_void_p
_i32 = C.c_int
_i64 = C.c_int64
_pi64 = C.POINTER(C.c_int64)
_pi32 = C.POINTER(C.c_int32)

# name -> (restype, argtypes); the complete exported surface of include/pagekv.h
SIGNATURES: dict[str, tuple] = {
    "pk_last_error": (C.c_char_p, []),
    "pk_abi_version": (_i32, []),
    "pk_pool_create": (_i32, [_i32, _i64, _i32, _i32, _i32, _i32, _i32, C.POINTER(_p)]),
    "pk_pool_destroy": (_i32, [_p]),
    "pk_pool_buffers": (_i32, [_p, C.POINTER(_p), C.POINTER(_p), _pi64]),
    "pk_pool_tc_info": (_i32, [_p, C.POINTER(_i32), C.POINTER(_i32), C.POINTER(_i32), C.POINTER(C.c_char_p)]),
    "pk_pool_copy_blocks": (_i32, [_p, _pi64, _i64, _p]),
    "pk_pool_copy_blocks_dev": (_i32, [_p, _p, _i64, _p]),
    "pk_pool_append": (_i32, [_p, _i32, _p, _p, _p, _i64, _p]),
    "pk_slot_mapping": (_i32, [_p, _i64, _p, _i64, _i32, _p, _p, _p]),
    "pk_batch_create": (_i32, [_p, C.POINTER(_p)]),
    "pk_batch_destroy": (_i32, [_p]),
    "pk_batch_plan": (_i32, [_p, _i32, _p, _p, _p, _p, _p, _p]),
    "pk_batch_rows": (_i32, [_p, C.POINTER(_p), C.POINTER(_p)]),
    "pk_batch_write_and_attend": (_i32, [_p, _i32, _i32, _p, _p, _p, _p, _p]),
    "pk_batch_attend": (_i32, [_p, _i32, _i32, _p, _p, _p]),
    "pk_batch_write_and_attend_host": (_i32, [_p, _i32, _i32, _p, _p, _p, _p, _p]),
    "pk_batch_check": (_i32, [_p, _p]),
    "pk_batch_stats": (_i32, [_p, _pi64]),
    "pk_batch_io_stats": (_i32, [_p, _pi64]),
    "pk_test_inject_launch_failure": (_i32, []),
    "pk_bm_truncate": (_i32, [_p, _i64, _i64]),
    "pk_batch_set_prefix_sharing": (_i32, [_p, _i32]),
    "pk_batch_prefix_stats": (_i32, [_p, _pi64]),
    "pk_plan_partition": (_i32, [_pi64, _i64, _i32, _i32, _pi64, C.POINTER(_i32)]),
    "pk_gather_interleave": (_i32, [_p, _p, _i32, _i64, _i64, _p]),
    "pk_peer_gather_create": (_i32, [_i32, _i32, _i32, _i64, C.POINTER(_p)]),
    "pk_peer_gather_handle": (_i32, [_p, C.c_char_p]),
    "pk_peer_gather_open": (_i32, [_p, C.c_char_p]),
    "pk_peer_gather_heads": (_i32, [_p, _p, _i64, _i64, C.POINTER(_p), _p]),
    "pk_peer_gather_write_and_attend": (_i32, [_p, _p, _i32, _i32, _p, _p, _p, C.POINTER(_p), _p]),
    "pk_peer_gather_check": (_i32, [_p, _p]),
    "pk_peer_gather_destroy": (_i32, [_p]),
    "pk_decode_attend_static": (_i32, [_p, _i32, _i32, _i32, _pi64, _pi32, _pi64, _p, _p, _p, _p]),
    "pk_selftest_bounded_wait": (_i32, [_i32, _i64, C.POINTER(_i32)]),
    "pk_batch_profile": (_i32, [_p, _i32]),
    "pk_batch_profile_read": (_i32, [_p, C.POINTER(C.c_double), _pi64]),
}

# block bookkeeping (host only)
SIGNATURES.update({
    "pk_bm_last_error": (C.c_char_p, []),
    "pk_bm_create": (C.c_int, [_i64, C.c_int, C.c_int, C.POINTER(_p)]),
    "pk_bm_destroy": (C.c_int, [_p]),
    "pk_bm_allocate_block": (C.c_int, [_p, _pi32]),
    "pk_bm_incref": (C.c_int, [_p, C.c_int32]),
    "pk_bm_decref": (C.c_int, [_p, C.c_int32]),
    "pk_bm_lookup": (C.c_int, [_p, C.c_char_p, _i64, _pi32]),
    "pk_bm_register": (C.c_int, [_p, C.c_int32, C.c_char_p, _i64]),
    "pk_bm_counts": (C.c_int, [_p, _pi64]),
    "pk_bm_refcounts": (C.c_int, [_p, C.POINTER(_pi64)]),
    "pk_bm_free_list": (C.c_int, [_p, _pi32, _i64, _pi64]),
    "pk_bm_evictable_list": (C.c_int, [_p, _pi32, _i64, _pi64]),
    "pk_bm_block_hash": (C.c_int, [_p, C.c_int32, C.c_char_p, _i64, _pi64]),
    "pk_bm_add_prefix_stats": (C.c_int, [_p, _i64, _i64]),
    "pk_bm_seq_allocate": (C.c_int, [_p, _i64, _i64, _pi32, _i64, C.c_char_p, _i64, _pi64]),
    "pk_bm_can_append": (C.c_int, [_p, _i64, _i64, C.POINTER(C.c_int)]),
    "pk_bm_ensure_capacity": (C.c_int, [_p, _i64, _i64, _i64, _pi64, _i64, _pi64]),
    "pk_bm_seq_hashes": (C.c_int, [_p, _i64, _pi64, C.c_char_p, _i64, _pi64]),
    "pk_bm_seq_hash_at": (C.c_int, [_p, _i64, _i64, C.c_char_p, _i64, _pi64]),
    "pk_bm_seq_push_hashes": (C.c_int, [_p, _i64, C.c_char_p, _i64, _i64]),
    "pk_bm_fork": (C.c_int, [_p, _i64, _i64]),
    "pk_bm_free_seq": (C.c_int, [_p, _i64]),
    "pk_bm_table": (C.c_int, [_p, _i64, _pi32, _i64, _pi64]),
    "pk_bm_seq_ids": (C.c_int, [_p, _pi64, _i64, _pi64]),
    "pk_bm_tables_csr": (C.c_int, [_p, _pi64, _i64, _pi64, _pi32, _i64, _pi64]),
})


class PagedKVError(RuntimeError):
    """A libpagekv call failed (status code in ``.status``)."""

    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


class DeviceTimeout(PagedKVError):
    """A bounded device-side wait gave up; the kernel returned early."""


_lib: C.CDLL | None = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Load (once) and type the library. Raises if it has not been built.

    The in-tree build is used unless ``PAGEKV_LIB`` names another libpagekv.so."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else Path(os.environ.get("PAGEKV_LIB", LIB_PATH))
    if not p.exists():
        raise ImportError(
            f"{p} is missing: build it with `python -m pagellm_b200.build` (nvcc, sm_100a)"
        )
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def last_error() -> str:
    return load().pk_last_error().decode(errors="replace")


def check(status: int) -> None:
    """Map a C status to the exception pagellm would raise for the same condition."""
    if status == PK_OK:
        return
    msg = last_error()
    if status == PK_ERR_OUT_OF_BLOCKS:
        from .cache.paged import OutOfBlocks

        raise OutOfBlocks(msg)
    if status in (PK_ERR_INVALID_ARG, PK_ERR_DUPLICATE):
        raise ValueError(msg)
    if status == PK_ERR_OUT_OF_RANGE:
        raise IndexError(msg)
    if status == PK_ERR_NOT_FOUND:
        raise KeyError(msg)
    if status == PK_ERR_TIMEOUT:
        raise DeviceTimeout(status, msg)
    if status == PK_ERR_DOUBLE_FREE:
        raise RuntimeError(msg)
    raise PagedKVError(status, msg)


def ptr(a) -> int:
    """Raw address of a torch tensor or numpy array (0 for None)."""
    if a is None:
        return 0
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data
