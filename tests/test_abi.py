"""The C ABI without a GPU: the library loads, exports exactly what include/pagekv.h
declares, and its host-only logic (argument checks, the split-KV partition) behaves."""

from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from pagellm_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "pagekv.h"


def declared() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^PK_API\s+[\w\s\*]*?\b(pk_\w+)\s*\(", text, flags=re.M))


def test_header_and_binding_agree():
    names = declared()
    assert len(names) >= 40
    assert names == set(_lib.SIGNATURES), names ^ set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), name
    assert lib.pk_abi_version() == 1


def test_pool_create_rejects_bad_arguments_before_touching_cuda():
    lib = _lib.load()
    h = C.c_void_p()
    assert lib.pk_pool_create(0, 10, 16, 2, 32, 0, 0, C.byref(h)) == _lib.PK_ERR_INVALID_ARG
    assert "positive" in _lib.last_error()
    assert lib.pk_pool_create(1, 10, 16, 2, 32, 7, 0, C.byref(h)) == _lib.PK_ERR_INVALID_ARG
    assert lib.pk_pool_create(1, 10, 16, 2, 32, 0, 0, None) == _lib.PK_ERR_INVALID_ARG
    assert lib.pk_batch_plan(None, 0, None, None, None, None, None, None) == _lib.PK_ERR_INVALID_ARG


@pytest.mark.parametrize("blocks,ctas", [([3, 1, 7, 2], 148), ([100] * 64, 148), ([144, 230, 31], 5),
                                         ([1], 148), (list(range(1, 300)), 148), ([2, 1] * 256, 148)])
def test_split_kv_partition_is_balanced_and_complete(blocks, ctas):
    """CTA c owns blocks [c*T/n, (c+1)*T/n): every block once, sizes differ by at most 1,
    n = max(1, min(max_ctas, T, max(T // 16, ceil(units / 3)))) so no CTA is empty, and a
    CTA gets 16 blocks or more unless the units are many and short."""
    lib = _lib.load()
    b = np.asarray(blocks, dtype=np.int64)
    T = int(b.sum())
    n = max(1, min(ctas, T, max(T // 16, -(-len(b) // 3))))
    first = np.zeros(n + 1, dtype=np.int64)
    got = C.c_int()
    assert lib.pk_plan_partition(b.ctypes.data_as(C.POINTER(C.c_int64)), len(b), ctas,
                                 first.ctypes.data_as(C.POINTER(C.c_int64)), C.byref(got)) == 0
    assert got.value == n and first[0] == 0 and first[-1] == T
    sizes = np.diff(first)
    assert sizes.min() == T // n and sizes.max() - sizes.min() <= 1
    if T // 16 >= -(-len(b) // 3):  # block-driven count
        assert sizes.min() >= min(T, 16)


def test_partition_rejects_empty_units():
    lib = _lib.load()
    b = np.array([2, 0, 3], dtype=np.int64)
    n = C.c_int()
    assert lib.pk_plan_partition(b.ctypes.data_as(C.POINTER(C.c_int64)), 3, 8, None, C.byref(n)) \
        == _lib.PK_ERR_INVALID_ARG
