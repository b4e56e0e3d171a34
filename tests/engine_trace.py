"""Engine traces recorded from pagellm's own LLMEngine (tests/golden/engine_*.npz, written by
``make_golden.py engine``): loading, and a replay through the CPU oracle.

A trace holds, per engine step, the copy-on-write copies made before the step's PagedBatch,
the batch's block tables, starts, n_new, attention mode, positions and slots, and (except for
structure-only traces) per layer the q / k / v the model passed to ``write_and_attend`` and
the output pagellm returned (pagellm engine/llm_engine.py:201-255).
"""

from __future__ import annotations

import json

import numpy as np
from conftest import load_npz

from oracle import paged_oracle as po


# float32 engine outputs: max |got - ref| <= 1e-5 x max |ref| over each layer's output. Both
# sides accumulate in float32 in different orders, so elements near zero carry absolute
# differences of ~1e-6 of the output's scale; a per-element relative bound would reject them.
F32_SCALED_RTOL = 1e-5


def assert_close_scaled(got, ref, rtol: float = F32_SCALED_RTOL):
    got, ref = np.asarray(got), np.asarray(ref)
    if ref.size == 0:
        return
    scale = float(np.max(np.abs(ref)))
    err = float(np.max(np.abs(got - ref)))
    assert err <= rtol * scale, f"max |diff| {err:.3e} > {rtol:g} x max |ref| {scale:.3e}"


class Step:
    def __init__(self, z: dict, i: int):
        ip, ids = z[f"s{i}_indptr"], z[f"s{i}_ids"]
        self.tables = [ids[ip[j]:ip[j + 1]].tolist() for j in range(len(ip) - 1)]
        self.copies = [tuple(map(int, c)) for c in z[f"s{i}_copies"]]
        self.starts = z[f"s{i}_starts"].tolist()
        self.n_new = z[f"s{i}_n_new"].tolist()
        paged, batch_decode = (int(x) for x in z[f"s{i}_mode"])
        self.attn = "paged" if paged else "gather"
        self.batch_decode = bool(batch_decode)
        self.positions = z[f"s{i}_positions"]
        self.slots = z[f"s{i}_slots"]
        self.q = z.get(f"s{i}_q")      # [layers][rows][H][d] float32, None for structure-only
        self.k = z.get(f"s{i}_k")
        self.v = z.get(f"s{i}_v")
        self.out = z.get(f"s{i}_out")

    @property
    def rows(self) -> int:
        return int(sum(self.n_new))


class Trace:
    def __init__(self, name: str):
        z = load_npz(f"engine_{name}.npz")
        self.name = name
        self.layers, self.H, self.KVH, self.d, self.num_blocks, self.bs = (int(x) for x in z["dims"])
        self.stats = json.loads(str(z["stats"]))
        self.steps = [Step(z, i) for i in range(int(z["nsteps"]))]


class OraclePool:
    """Host pool ``[layers][num_blocks][bs][kvh][d]`` (zero-filled, as pagellm's) driven
    through the oracle; ``bf16`` rounds every appended row as a bf16 pool stores it."""

    def __init__(self, layers, num_blocks, bs, kvh, d, bf16: bool = False):
        self.k = np.zeros((layers, num_blocks, bs, kvh, d), np.float32)
        self.v = np.zeros_like(self.k)
        self.bs, self.bf16 = bs, bf16

    def step(self, st: Step, layer_inputs):
        """Copies, then every layer: yields (layer, oracle output)."""
        po.copy_blocks(self.k, self.v, st.copies)
        meta = po.StepMeta(st.tables, st.starts, st.n_new, self.bs, st.batch_decode, st.attn)
        for layer, (q, k, v) in enumerate(layer_inputs):
            if self.bf16:
                k, v = po.bf16_round(k), po.bf16_round(v)
            kf = self.k[layer].reshape(-1, *self.k.shape[3:])
            vf = self.v[layer].reshape(-1, *self.v.shape[3:])
            yield layer, po.write_and_attend(kf, vf, meta, q, k, v, self.k[layer], self.v[layer])
