"""Shared fixtures. GPU tests carry ``@pytest.mark.gpu``; everything else runs on CPU."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture
def rng() -> np.random.Generator:
    return np.random.default_rng(1234)


def load_npz(name: str) -> dict:
    with np.load(GOLDEN / name) as z:
        return {k: z[k] for k in z.files}


def load_traces() -> list:
    return json.loads((GOLDEN / "allocator_traces.json").read_text())


def bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << np.uint32(16)).view(np.float32)


def step_inputs(case: dict) -> dict:
    """Decode a ``step_*.npz`` fixture into float32 arrays and per-sequence tables."""
    H, KVH, d, bs, nb = (int(x) for x in case["dims"])
    out = dict(H=H, KVH=KVH, d=d, bs=bs, num_blocks=nb)
    bf16 = case["kc"].dtype == np.uint16
    for key in ("kc", "vc", "k", "v"):
        out[key] = bf16_bits_to_f32(case[key]) if bf16 else case[key]
    out["bf16"] = bf16
    ip, ids = case["indptr"], case["ids"]
    out["tables"] = [ids[ip[i]:ip[i + 1]].tolist() for i in range(len(ip) - 1)]
    for key in ("starts", "n_new", "ctx_slots", "q", "positions", "slots", "out"):
        out[key] = case[key]
    return out
