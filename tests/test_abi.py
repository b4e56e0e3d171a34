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


def _partition(blocks, ctas, switch):
    lib = _lib.load()
    b = np.asarray(blocks, dtype=np.int64)
    T = int(b.sum())
    n = max(1, min(ctas, T, max(T // 16, -(-len(b) // 3))))
    first = np.full(n + 1, -1, dtype=np.int64)
    got = C.c_int()
    assert lib.pk_plan_partition(b.ctypes.data_as(C.POINTER(C.c_int64)), len(b), ctas, switch,
                                 first.ctypes.data_as(C.POINTER(C.c_int64)), C.byref(got)) == 0
    return T, n, first[:got.value + 1], got.value


def _range_cost(bounds, b, e, switch):
    """Blocks of [b, e) plus `switch` per unit boundary strictly inside it."""
    return (e - b) + switch * int(np.count_nonzero((bounds > b) & (bounds < e)))


def _optimum(blocks, n, switch):
    """Smallest achievable largest range cost with at most n non-empty ranges (exact DP)."""
    ub = np.concatenate([[0], np.cumsum(blocks)])
    T, inner = int(ub[-1]), ub[1:-1]
    inf = float("inf")
    best = [0.0] + [inf] * T  # best[e]: min max cost covering [0, e) with k ranges
    out = inf
    for _ in range(n):
        nxt = [inf] * (T + 1)
        for e in range(1, T + 1):
            nxt[e] = min((max(best[b], _range_cost(inner, b, e, switch)) for b in range(e) if best[b] < inf),
                         default=inf)
        best = nxt
        out = min(out, best[T])
    return out


@pytest.mark.parametrize("blocks,ctas", [([3, 1, 7, 2], 148), ([100] * 64, 148), ([144, 230, 31], 5),
                                         ([1], 148), (list(range(1, 300)), 148), ([2, 1] * 256, 148)])
@pytest.mark.parametrize("switch", [0, 6])
def test_split_kv_partition_is_complete(blocks, ctas, switch):
    """Every block once in contiguous, non-empty CTA ranges, at most
    n = max(1, min(max_ctas, T, max(T // 16, ceil(units / 3)))) of them; with no unit cost
    the largest range is ceil(T / n) blocks, the least possible."""
    T, n, first, used = _partition(blocks, ctas, switch)
    assert 1 <= used <= n and first[0] == 0 and first[-1] == T
    assert np.all(np.diff(first) > 0)
    if switch == 0:
        assert np.diff(first).max() == -(-T // n)


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("switch", [0, 2, 6])
def test_split_kv_partition_minimises_the_largest_cost(seed, switch):
    """The cut's largest cost (blocks + switch per unit boundary inside a range) equals the
    optimum over all cuts into at most n ranges, found by exhaustive dynamic programming."""
    rng = np.random.default_rng(seed)
    blocks = rng.integers(1, 25, rng.integers(2, 9)).tolist()
    ctas = int(rng.integers(2, 7))
    T, n, first, used = _partition(blocks, ctas, switch)
    inner = np.cumsum(blocks)[:-1]
    worst = max(_range_cost(inner, int(first[c]), int(first[c + 1]), switch) for c in range(used))
    assert worst == _optimum(blocks, n, switch), (blocks, n, switch, first)


def test_partition_rejects_empty_units():
    lib = _lib.load()
    b = np.array([2, 0, 3], dtype=np.int64)
    n = C.c_int()
    assert lib.pk_plan_partition(b.ctypes.data_as(C.POINTER(C.c_int64)), 3, 8, 0, None, C.byref(n)) \
        == _lib.PK_ERR_INVALID_ARG
    ok = np.array([2, 1, 3], dtype=np.int64)
    assert lib.pk_plan_partition(ok.ctypes.data_as(C.POINTER(C.c_int64)), 3, 8, -1, None, C.byref(n)) \
        == _lib.PK_ERR_INVALID_ARG


def test_host_array_addresses():
    """The Python surface passes numpy buffers to the C ABI by address: the buffer-protocol
    route for writable arrays, ndarray.ctypes for read-only and empty ones; all agree."""
    import pagellm_b200.cache.paged as paged

    a = np.arange(10, dtype=np.int64)
    assert paged._addr(a) == a.ctypes.data
    ro = np.arange(6, dtype=np.int32)
    ro.setflags(write=False)
    assert paged._addr(ro) == ro.ctypes.data
    empty = np.zeros(0, dtype=np.int32)
    assert paged._addr(empty) == empty.ctypes.data
    sub = np.arange(16, dtype=np.float32)[4:]
    assert paged._addr(sub) == sub.ctypes.data
