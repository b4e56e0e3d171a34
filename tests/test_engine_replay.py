"""pagellm's own serving engine, replayed through pagellm_b200.cache on the GPU.

The fixtures (tests/golden/engine_*.npz) were recorded by running pagellm's LLMEngine with
its bundled 4-layer model (make_golden.py ``engine_trace``): for every engine step, the
copy-on-write copies made before it, the PagedBatch it built and, per layer, the q / k / v
the model handed to ``write_and_attend`` and the output pagellm returned. Here the same
calls go to the device pool, in the same order, as LLMEngine.step would make them with
this package's ``PagedKVPool`` / ``PagedBatch`` swapped in (engine/llm_engine.py:201-228):

* float32 pool, the bundled model's shape: positions and slots bit-exact, every layer's
  output within 1e-5 of its scale of pagellm's, and after the last step the whole device
  pool (every layer, every block) equal bit for bit to the oracle's replay of the trace
  (append and copy-on-write are exact);
* the step structure of a run with 16-token blocks (forks sharing prompt blocks, prefix
  hits, chunked prefill, decodes) at a tensor-core shape (bf16, 8 query heads over 2 KV
  heads, head_dim 128) with seeded inputs: every layer's output against the oracle within
  the bf16 tolerance (2e-2 max-abs), with the shared-prefix pass off, on a cost estimate,
  and forced; the pool bit for bit against the oracle's at the end.
"""

from __future__ import annotations

import numpy as np
import pytest
from engine_trace import OraclePool, Trace, assert_close_scaled
from gpu_util import Shape, torch_cuda

pytestmark = pytest.mark.gpu

BF16_ATOL = 2e-2


@pytest.mark.parametrize("name", ["serve", "preempt", "chunked"])
def test_pagellm_engine_trace_fp32(name):
    torch = torch_cuda()
    from pagellm_b200.cache import PagedBatch, PagedKVPool

    tr = Trace(name)
    pool = PagedKVPool(Shape(tr.layers, tr.KVH, tr.d), tr.num_blocks, tr.bs, np.float32)
    oracle = OraclePool(tr.layers, tr.num_blocks, tr.bs, tr.KVH, tr.d)
    for st in tr.steps:
        pool.copy_blocks(st.copies)  # LLMEngine.step: pool.copy_block for each scheduled copy
        b = PagedBatch(pool, st.tables, st.starts, st.n_new, st.attn, st.batch_decode)
        np.testing.assert_array_equal(b.positions, st.positions)
        np.testing.assert_array_equal(b.slots, st.slots)
        for li in range(tr.layers):
            out = b.write_and_attend(li, st.q[li], st.k[li], st.v[li])
            assert out.dtype == np.float32 and out.shape == st.out[li].shape
            assert_close_scaled(out, st.out[li])
        b.check()
        for _ in oracle.step(st, [(st.q[li], st.k[li], st.v[li]) for li in range(tr.layers)]):
            pass
    torch.cuda.synchronize()
    np.testing.assert_array_equal(pool.k.cpu().numpy(), oracle.k)
    np.testing.assert_array_equal(pool.v.cpu().numpy(), oracle.v)


@pytest.mark.parametrize("mode", ["off", "auto", "always"])
def test_engine_structure_bf16_tensor_core_shape(mode):
    torch = torch_cuda()
    from pagellm_b200.cache import PagedBatch, PagedKVPool

    tr = Trace("serve16")
    layers, H, KVH, d = 2, 8, 2, 128
    pool = PagedKVPool(Shape(layers, KVH, d), tr.num_blocks, tr.bs, "bfloat16")
    assert pool.tensor_core_path[0], pool.tensor_core_path[1]
    oracle = OraclePool(layers, tr.num_blocks, tr.bs, KVH, d, bf16=True)
    rng = np.random.default_rng(3)
    seen = {"wide": 0, "groups": 0, "tc_units": 0}
    for st in tr.steps:
        pool.copy_blocks(st.copies)
        b = PagedBatch(pool, st.tables, st.starts, st.n_new)
        b.prefix_sharing = mode
        np.testing.assert_array_equal(b.slots, st.slots)
        inputs = [(rng.standard_normal((st.rows, H, d), dtype=np.float32),
                   rng.standard_normal((st.rows, KVH, d), dtype=np.float32),
                   rng.standard_normal((st.rows, KVH, d), dtype=np.float32)) for _ in range(layers)]
        got = [b.write_and_attend(li, *inputs[li]) for li in range(layers)]
        b.check()
        s = b.stats()
        seen["wide"] += s["wide_items"]
        seen["tc_units"] += s["tc_units"]
        seen["groups"] += b.prefix_stats()["groups"]
        for li, ref in oracle.step(st, inputs):
            err = float(np.max(np.abs(got[li] - ref)))
            assert err <= BF16_ATOL, (li, err)
    torch.cuda.synchronize()
    bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    from oracle import paged_oracle as po

    assert np.array_equal(bits(pool.k), po.bf16_bits(oracle.k))
    assert np.array_equal(bits(pool.v), po.bf16_bits(oracle.v))
    # the replay reached the tcgen05 chunk kernel and the split-KV kernel, and, unless off,
    # the shared-prefix pass over forks / prefix hits
    assert seen["wide"] > 0 and seen["tc_units"] > 0, seen
    assert (seen["groups"] > 0) == (mode != "off") or mode == "auto", seen
