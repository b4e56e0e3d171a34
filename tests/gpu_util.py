"""Helpers for the GPU parity tests: device pools filled with seeded data and the CPU
oracle run on exactly the values the device holds."""

from __future__ import annotations

import numpy as np

from oracle import paged_oracle as po


class Shape:
    def __init__(self, n_layers, n_kv_heads, head_dim):
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim


def torch_cuda():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def make_pool(w, seed: int = 0, layers: int = 1):
    """Device pool for workload ``w`` with every slot of every layer ~ N(0, 1)."""
    torch = torch_cuda()
    from pagellm_b200.cache import PagedKVPool

    pool = PagedKVPool(Shape(layers, w.KVH, w.D), w.num_blocks, w.bs,
                       "bfloat16" if w.dtype == "bf16" else np.float32)
    g = torch.Generator(device="cuda").manual_seed(seed)
    for t in (pool.k, pool.v):
        for li in range(layers):
            t[li].copy_(torch.randn(t[li].shape, generator=g, device="cuda").to(t.dtype))
    return pool


def step_inputs(w, seed: int = 1):
    torch = torch_cuda()
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((w.rows, w.H, w.D), generator=g, device="cuda")
    k = torch.randn((w.rows, w.KVH, w.D), generator=g, device="cuda")
    v = torch.randn((w.rows, w.KVH, w.D), generator=g, device="cuda")
    return q, k, v


def gather_rows(pool, layer: int, slots: np.ndarray):
    """float32 numpy copy of pool rows (slot order) for K and V."""
    torch = torch_cuda()
    idx = torch.as_tensor(np.asarray(slots, np.int64), device=pool.device)
    k = pool.k_flat[layer].index_select(0, idx).float().cpu().numpy()
    v = pool.v_flat[layer].index_select(0, idx).float().cpu().numpy()
    return k, v


def oracle_rows(pool, w, seqs, q_host, layer: int = 0):
    """Oracle attention output for sequences ``seqs`` of workload ``w``, reading the
    device pool as it is now (after the step's append): {seq: (row_slice, out)}."""
    res = {}
    offs = np.concatenate([[0], np.cumsum(w.n_new)])
    for i in seqs:
        s, n = int(w.starts[i]), int(w.n_new[i])
        ctx = po.slot_mapping(w.tables[i], np.arange(s + n), w.bs)
        kc, vc = gather_rows(pool, layer, ctx)
        a, b = int(offs[i]), int(offs[i + 1])
        res[i] = (slice(a, b), po.attention_dense(q_host[a:b], kc, vc, s))
    return res


def bf16_bits_of_tensor(t) -> np.ndarray:
    torch = torch_cuda()
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
