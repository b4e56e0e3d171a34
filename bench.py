"""Benchmark of the paged KV-cache hot path on B200: decode-attention tokens/s and HBM GB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

One step = one layer of ``PagedBatch.write_and_attend`` for the workload (append the new
K/V rows through the slot mapping, then split-KV GQA attention over the paged cache) on
seeded synthetic inputs; default workload C2 (Llama-3-8B shape, batch 64, bf16 K/V,
contexts U{512..4096}).

* ``value``: tokens/s over all ranks, K steps timed with CUDA events (inputs resident).
  Under torchrun every rank runs the same C2 batch on its own pool (sequence-sharded, no
  collective on the data path): weak scaling.
* ``e2e``: the same through the public Python API from pinned HOST buffers, every step
  re-planning the batch (block tables up), q/k/v up and the output down.
* ``roofline``: the dominant kernel's algorithmic bytes (split-KV decode) or FLOPs (the
  tcgen05 wide-tile pass, C3/C4) per event-timed launch against the measured HBM copy
  bandwidth or sustained bf16 throughput (MEASURED_PEAKS.json).
* ``c5``: the 70B-shaped long-context batch (128 sequences) split over the N ranks of this
  run, strong scaling, in both multi-GPU layouts: sequence-sharded (whole sequences per GPU,
  longest first, no collective) and head-sharded (KV heads per GPU, NCCL all-gather of the
  output slices plus the interleave kernel inside every step). At least 200 steps each.
* ``configs`` (one GPU only): C1, C3, C4 measured the same way as ``value``.
* ``cpu_baseline``: the CPU oracle (numpy restatement of pagellm's gather path) on a
  bounded sample of the same workload on this host.

``--impl reference`` times pagellm's own numpy path (``PagedBatch.write_and_attend`` from
the install in baseline/_ref; the oracle port when that is absent) on this host's cores on
the same workload, rank 0 only (other ranks exit).
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode-attn tokens/s & achieved HBM GB/s (% of 8 TB/s) at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1400.0  # sustained under the power cap
# dram__bytes_read.sum + dram__bytes_write.sum of one tc_attn_kernel launch on the default
# C2 workload (620,258,304 + 6,978,304), from an ncu --set full capture of this kernel (one
# launch, cold L2); every rank runs the same batch, so it holds at every N
TC_C2_NCU_TRAFFIC = 627_236_608
TC_C2_NCU_SOURCE = "ncu capture of one tc_attn_kernel launch on this workload (cold L2): dram read + write bytes"
C5_MIN_STEPS = 200
RESULT_OUT = sys.stdout

WORKLOAD_TEXT = {
    "c1": "fp32 decode B=8 H=4 KVH=2 d=32 bs=16 L~U{1..256}",
    "c2": "Llama-3-8B decode attention, 1 layer, B=64 H=32 KVH=8 d=128 bs=16, L~U{512..4096}, bf16 K/V fp32 accumulate",
    "c3": "mixed step: 16 decodes L~U{256..2048} + 512-query chunk at 1024..1535",
    "c4": "64 requests x 4 forks share a 2048-token prefix, 192 CoW copies, 5-token verify",
    "c5": "70B long-context decode B=128 H=64 KVH=8 d=128, L~lognormal(8192,0.75) clip[1024,32768]",
}
KERNEL_NAMES = {1: "tc_attn_kernel (split-KV paged attention, TMA + mma.sync bf16)",
                3: "generic_attn_kernel (CUDA cores)",
                4: "wide_attn_kernel (tcgen05/TMEM chunk attention, TMA)"}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    """Dense bf16 TFLOP/s for a kernel timed inside a long step: the sustained figure."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured (sustained)"
    return FALLBACK_BF16_TFLOPS, "fallback"


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples of SM clock / throttle reasons while GPU work runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.rows, self.proc = gpu, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi's first query initialises NVML, which can stall the GPU for a while
            # on a fresh box: let that happen before any timed work
            t0 = time.time()
            while not self.rows and time.time() - t0 < 10.0 and self.proc.poll() is None:
                time.sleep(0.02)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 9:
                self.rows.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def mark(self) -> int:
        return len(self.rows)

    def summary(self, since: int = 0):
        rows = self.rows[since:]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1])]
        mx = [num(r[2]) for r in rows if num(r[2])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------------ CPU path
def cpu_inputs(w, seqs, seed: int = 0):
    """Compact host pool holding exactly the blocks of sequences ``seqs`` of workload ``w``
    (K/V ~ N(0,1), bf16-rounded for bf16 workloads) and the step's q/k/v for them."""
    from oracle import paged_oracle as po

    rng = np.random.default_rng(seed)
    bs, kvh, d = w.bs, w.KVH, w.D
    remap: dict[int, int] = {}  # workload block id -> compact id (shared blocks stay shared)
    tables = []
    for i in seqs:
        tables.append([remap.setdefault(int(b_), len(remap)) for b_ in w.tables[i]])
    nb = len(remap)
    pairs = [(remap[s_], remap[d_]) for s_, d_ in w.cow_pairs if s_ in remap and d_ in remap]
    kp = rng.standard_normal((nb * bs, kvh, d), dtype=np.float32)
    vp = rng.standard_normal((nb * bs, kvh, d), dtype=np.float32)
    starts = [int(w.starts[i]) for i in seqs]
    n_new = [int(w.n_new[i]) for i in seqs]
    rows = sum(n_new)
    q = rng.standard_normal((rows, w.H, d), dtype=np.float32)
    k = rng.standard_normal((rows, kvh, d), dtype=np.float32)
    v = rng.standard_normal((rows, kvh, d), dtype=np.float32)
    if w.dtype == "bf16":
        kp, vp, k, v = (po.bf16_round(a) for a in (kp, vp, k, v))
    return dict(kp=kp, vp=vp, nb=nb, tables=tables, pairs=pairs, starts=starts, n_new=n_new, rows=rows,
                q=q, k=k, v=v)


def cpu_reference(w, sample_seqs: int, min_seconds: float, max_reps: int, seed: int = 0):
    """The oracle's numpy port of pagellm's gather path (append + padded batched decode)
    on ``sample_seqs`` sequences of workload ``w``; K/V bf16-rounded for bf16 workloads.
    Runs until ``min_seconds`` have passed or ``max_reps`` steps (at least one).
    Returns (tokens/s, seconds, reps, threads)."""
    from oracle import paged_oracle as po

    x = cpu_inputs(w, list(range(min(sample_seqs, w.nseq))), seed)
    meta = po.StepMeta(x["tables"], x["starts"], x["n_new"], w.bs)
    po.write_and_attend(x["kp"], x["vp"], meta, x["q"], x["k"], x["v"])  # warm-up
    t0 = time.perf_counter()
    reps = 0
    while reps < max(1, max_reps) and (reps == 0 or time.perf_counter() - t0 < min_seconds):
        meta = po.StepMeta(x["tables"], x["starts"], x["n_new"], w.bs)
        po.write_and_attend(x["kp"], x["vp"], meta, x["q"], x["k"], x["v"])
        reps += 1
    dt = time.perf_counter() - t0
    threads = int(os.environ.get("OPENBLAS_NUM_THREADS") or os.environ.get("OMP_NUM_THREADS") or os.cpu_count())
    return x["rows"] * reps / dt, dt, reps, threads


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ------------------------------------------------------------------------------ GPU path
class Ctx:
    """Rank, device, process group and the timing helpers of one bench process."""

    def __init__(self):
        import torch
        import torch.distributed as dist

        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            from datetime import timedelta

            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=self.dev)
        self.stream = torch.cuda.current_stream(self.dev)
        self.st = self.stream.cuda_stream

    def flush_l2(self):
        """Evict L2 with a 256 MB write on the launching stream."""
        if not hasattr(self, "_flush"):
            self._flush = self.torch.empty(64 << 20, dtype=self.torch.float32, device=self.dev)
        self._flush.fill_(1.0)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize(self.dev)

    def max_over_ranks(self, x: float) -> float:
        if self.world == 1:
            return x
        t = self.torch.tensor([x], device=self.dev, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(self, x: float) -> float:
        if self.world == 1:
            return x
        t = self.torch.tensor([x], device=self.dev, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return float(t.item())

    def timed_flushed(self, fn, steps: int, warmup: int) -> float:
        """Milliseconds for ``steps`` calls of ``fn`` with L2 flushed before each: every call is
        timed alone (CUDA events on the launching stream) after a 256 MB write that evicts the
        126 MB L2, and the per-call times are summed (the flushes are not counted)."""
        torch = self.torch
        for _ in range(warmup):
            fn()
        self.barrier()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for e0, e1 in evs:
            self.flush_l2()
            e0.record(self.stream)
            fn()
            e1.record(self.stream)
        self.barrier()
        return self.max_over_ranks(sum(e0.elapsed_time(e1) for e0, e1 in evs))

    def timed(self, fn, steps: int, warmup: int) -> float:
        """Milliseconds for ``steps`` calls of ``fn`` (after ``warmup`` untimed ones), CUDA
        events on the launching stream, barrier + synchronize on both sides, max over ranks."""
        torch = self.torch
        for _ in range(warmup):
            fn()
        self.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for _ in range(steps):
            fn()
        e1.record(self.stream)
        self.barrier()
        return self.max_over_ranks(e0.elapsed_time(e1))


class Job:
    """One workload on this rank: pool filled with N(0,1) K/V, the step's batch and
    device-resident q/k/v/out."""

    def __init__(self, ctx: Ctx, w, seed: int = 0):
        from pagellm_b200 import _lib
        from pagellm_b200.cache import PagedBatch, PagedKVPool

        torch = ctx.torch
        self.ctx, self.w = ctx, w

        class Shape:
            n_layers, n_kv_heads, head_dim = 1, w.KVH, w.D

        self.pool = PagedKVPool(Shape, w.num_blocks, w.bs, "bfloat16" if w.dtype == "bf16" else np.float32)
        g = torch.Generator(device=ctx.dev).manual_seed(seed)
        for t in (self.pool.k, self.pool.v):
            t[0].copy_(torch.randn(t[0].shape, generator=g, device=ctx.dev).to(t.dtype))
        self.pairs_dev = None
        if w.cow_pairs:
            self.pairs_dev = torch.as_tensor(np.asarray(w.cow_pairs, dtype=np.int64).reshape(-1, 2), device=ctx.dev)
            self.pool.copy_blocks(w.cow_pairs)
        self.indptr, self.ids = w.csr()
        self.batch = PagedBatch(self.pool, (self.indptr, self.ids), w.starts, w.n_new)
        self.q = torch.randn((w.rows, w.H, w.D), generator=g, device=ctx.dev)
        self.k = torch.randn((w.rows, w.KVH, w.D), generator=g, device=ctx.dev)
        self.v = torch.randn((w.rows, w.KVH, w.D), generator=g, device=ctx.dev)
        self.out = torch.empty_like(self.q)
        self.lib = _lib.load()
        self._check = _lib.check

    def attend_layer(self):
        rc = self.lib.pk_batch_write_and_attend(self.batch._b, 0, self.w.H, self.q.data_ptr(), self.k.data_ptr(),
                                                self.v.data_ptr(), self.out.data_ptr(), self.ctx.st)
        if rc:
            self._check(rc)

    def step(self):
        """The workload's step: its copy-on-write copies (C4's forks), then the layer."""
        if self.pairs_dev is not None:
            rc = self.lib.pk_pool_copy_blocks_dev(self.pool.handle, self.pairs_dev.data_ptr(), len(self.pairs_dev),
                                                  self.ctx.st)
            if rc:
                self._check(rc)
        self.attend_layer()

    def launches_per_step(self) -> int:
        return self.batch.stats()["launches"] + (1 if self.pairs_dev is not None else 0)

    def profile(self, fn, steps: int, flush=None):
        """Per-kernel averages (ms per launch, launches) over ``steps`` calls of ``fn``,
        events recorded by the library on the launching stream around each launch; ``flush``
        (if given) runs before every call, outside the recorded launches."""
        lib = self.lib
        lib.pk_batch_profile(self.batch._b, 1)
        for _ in range(steps):
            if flush is not None:
                flush()
            fn()
        ms = (C.c_double * 5)()
        n = (C.c_int64 * 5)()
        self._check(lib.pk_batch_profile_read(self.batch._b, ms, n))
        lib.pk_batch_profile(self.batch._b, 0)
        return list(ms), list(n)

    def close(self):
        self.batch = None
        self.pool.close()


def attention_roofline(w, batch, prof_ms, prof_n, traffic=None):
    """Roofline object for the dominant attention kernel of a step of ``w``."""
    uniq = w.unique_kv_bytes()
    alg = (uniq + w.rows * w.H * w.D * 8 + int(sum(-(-int(L) // w.bs) for L in w.ctx_lens)) * 4 + w.nseq * 12)
    # the wide-tile (tensor) kernel whenever the step has one (its split-KV kernel can take as
    # long on C3, and the line should not flip between HBM and tensor rooflines run to run),
    # else the longest of the others
    kind = 4 if prof_n[4] else max((1, 3), key=lambda i: prof_ms[i])
    avg_ms = prof_ms[kind] / max(1, prof_n[kind])
    hbm, hbm_src = peaks()
    achieved = alg / (avg_ms / 1e3) / 1e9
    r = {
        "bound": "hbm", "kernel": KERNEL_NAMES[kind], "achieved": round(achieved, 1), "peak": hbm,
        "unit": "GB/s", "frac": round(achieved / hbm, 4), "peak_source": hbm_src, "traffic": traffic,
        "algorithmic_bytes_per_launch": alg, "avg_launch_us": round(avg_ms * 1e3, 2),
        "kernel_us": {nm: round(prof_ms[i] / max(1, prof_n[i]) * 1e3, 2)
                      for i, nm in enumerate(("append", "tc_attention", "merge", "cuda_core_attention",
                                              "wide_tcgen05_attention")) if prof_n[i]},
    }
    if kind == 4:
        # compute-bound wide-tile pass: its algorithmic FLOPs (Q.K^T + P.V over the keys each
        # row sees): the causal chunks it takes (>= 64 query rows per KV head) plus the
        # shared-prefix pass
        g = w.H // w.KVH
        chunk_tk = sum(sum(int(w.starts[i]) + t + 1 for t in range(int(w.n_new[i])))
                       for i in range(w.nseq) if int(w.n_new[i]) * g >= 64)
        flops = 4.0 * w.H * w.D * (chunk_tk + batch.prefix_stats()["token_keys"])
        tp, tp_src = tensor_peak()
        tflops = flops / (avg_ms / 1e3) / 1e12
        r.update({"bound": "tensor", "achieved": round(tflops, 1), "peak": tp, "unit": "TFLOP/s",
                  "frac": round(tflops / tp, 4), "peak_source": tp_src, "traffic": None,
                  "algorithmic_flops_per_launch": flops, "algorithmic_bytes_per_launch": None})
    return r, kind


def measure_c5(ctx: Ctx, layout: str, steps: int, warmup: int) -> dict:
    """C5 (128 sequences) split over this run's ranks, one layout, strong scaling."""
    from pagellm_b200 import workloads
    from pagellm_b200.sharding import HeadGather, PeerHeadGather, shard_sequences

    torch = ctx.torch
    L = workloads.c5_lengths(0)
    if layout == "head":
        if 8 % ctx.world:
            return {"skipped": f"8 KV heads do not split over {ctx.world} ranks"}
        w = workloads.c5(0, lengths=L, kv_heads=8 // ctx.world)
    else:
        w = workloads.c5(0, lengths=L[shard_sequences(L, ctx.world)[ctx.rank]])
    job = Job(ctx, w, seed=ctx.rank)
    sharded = layout == "head" and ctx.world > 1
    # head-sharded: PeerHeadGather.write_and_attend's default for this world size (the
    # exchange inside the attention kernel at 2 ranks, attention + one push launch beyond);
    # the other form, and the NCCL all-gather + interleave kernel, are timed beside it
    gather = PeerHeadGather() if sharded else None
    nccl = HeadGather() if sharded else None
    full = {}

    def step():
        if gather is not None:
            full["out"] = gather.write_and_attend(job.batch, 0, job.q, job.k, job.v)
        else:
            job.attend_layer()

    ms = ctx.timed(step, steps, warmup)
    us = ms / steps * 1e3
    if sharded:
        gather.check()
        out_ref = full["out"].clone()
        alt = ctx.world > 2  # the form the default does not use: fused beyond 2 ranks
        fused_out = gather.write_and_attend(job.batch, 0, job.q, job.k, job.v, fused=alt).clone()
        gather.check()
        job.attend_layer()
        same = bool(torch.equal(out_ref, nccl(job.out))) and bool(torch.equal(fused_out, out_ref))
        ms_alt = ctx.timed(lambda: gather.write_and_attend(job.batch, 0, job.q, job.k, job.v, fused=alt),
                           steps, warmup)
        gather.check()
        ms_nccl = ctx.timed(lambda: (job.attend_layer(), nccl(job.out)), steps, warmup)
    prof_ms, prof_n = job.profile(job.attend_layer, steps)
    ctx.barrier()
    kernel_us = ctx.max_over_ranks(prof_ms[1] / max(1, prof_n[1]) * 1e3)
    res = {
        "layout": ("head-sharded: 8/N KV heads of every sequence per GPU; each GPU's [128, 64/N, 128] fp32 "
                   "output is stored into every GPU's [128, 64, 128] result over peer memory, by the "
                   "attention kernel itself at 2 GPUs, by one push launch after it beyond (epoch flags)")
        if layout == "head" else "sequence-sharded: whole sequences per GPU (longest first), no collective",
        "steps": steps,
        "us_per_step": round(us, 2),
        "tokens_per_s": round(len(L) * steps / (ms / 1e3), 1),
        "attention_kernel_us": round(kernel_us, 2),
    }
    if sharded:
        gms = ctx.timed(lambda: gather(job.out), steps, 3)
        nms = ctx.timed(lambda: nccl(job.out), steps, 3)
        res["push_us"] = round(gms / steps * 1e3, 2)
        res["other_exchange_path"] = {"us_per_step": round(ms_alt / steps * 1e3, 2),
                                      "what": ("the exchange inside the attention kernel (one launch per step)" if alt
                                               else "attention, then one push launch")}
        res["nccl_allgather_path"] = {"us_per_step": round(ms_nccl / steps * 1e3, 2),
                                      "gather_us": round(nms / steps * 1e3, 2)}
        res["results_equal_across_paths"] = same
        gather.close()
    kv = ctx.sum_over_ranks(float(w.kv_read_bytes()))
    hbm, src = peaks()
    per_gpu = kv / ctx.world / (us / 1e6) / 1e9
    res.update({
        "kv_bytes_per_step_all_gpus": int(kv),
        "hbm_gbs_per_gpu": round(per_gpu, 1),
        "hbm_frac_per_gpu": round(per_gpu / hbm, 4),
        "peak_source": src,
        "context_tokens_per_gpu_max": int(ctx.max_over_ranks(float(w.ctx_lens.sum()))),
        "context_tokens_all_gpus": int(L.sum()),
        "launches_per_step": job.launches_per_step() + (1 if sharded and ctx.world > 2 else 0),
    })
    assert torch.isfinite(job.out).all()
    job.close()
    return res


def measure_config(ctx: Ctx, name: str, steps: int, warmup: int) -> dict:
    """One single-GPU config line: rows/s with inputs resident and the dominant kernel's
    roofline."""
    from pagellm_b200 import workloads

    w = workloads.make(name, seed=0)
    job = Job(ctx, w)
    fits = w.unique_kv_bytes() <= 126e6
    # a step whose distinct K/V fits in L2 is timed with L2 flushed before it, as after
    # another layer's step
    ms = ctx.timed_flushed(job.step, steps, warmup) if fits else ctx.timed(job.step, steps, warmup)
    prof_ms, prof_n = job.profile(job.step, steps, flush=ctx.flush_l2 if fits else None)
    roof, _ = attention_roofline(w, job.batch, prof_ms, prof_n)
    res = {
        "workload": f"{name}: {WORKLOAD_TEXT[name]}",
        "value": round(w.rows * steps / (ms / 1e3), 1),
        "unit": "query rows/s" if name in ("c3", "c4") else "tokens/s",
        "steps": steps,
        "ms_per_step": round(ms / steps, 5),
        "rows_per_step": w.rows,
        "step_gbs": round(w.algorithmic_bytes() / (ms / steps / 1e3) / 1e9, 1),
        "attention_tflops": round(w.attention_flops() / (ms / steps / 1e3) / 1e12, 2),
        "cow_pairs_per_step": len(w.cow_pairs),
        "prefix_stats": job.batch.prefix_stats(),
        "l2": "inputs larger than L2" if not fits
              else "distinct K/V per step fits in L2 (126 MB): L2 flushed (256 MB write) before every timed step",
        "launches_per_step": job.launches_per_step(),
        "roofline": roof,
    }
    job.close()
    return res


def run_ours(args):
    from pagellm_b200 import workloads
    from pagellm_b200.cache import PagedBatch

    ctx = Ctx()
    torch = ctx.torch
    warmup = max(args.warmup, 3)
    # every rank runs the same batch (seed 0) on its own pool: weak scaling whose efficiency
    # measures interference only
    w = workloads.make(args.config, seed=0)
    job = Job(ctx, w, seed=0)

    fits = w.unique_kv_bytes() <= 126e6  # L2-resident step: flush L2 before each timed step
    with ClockSampler(ctx.local) as clocks:
        ms = ctx.timed_flushed(job.step, args.steps, warmup) if fits else ctx.timed(job.step, args.steps, warmup)
        clk = clocks.summary()
        job.batch.check()
        launches_per_step = job.launches_per_step()
        prof_ms, prof_n = job.profile(job.step, args.steps, flush=ctx.flush_l2 if fits else None)
        ctx.barrier()

        # end to end through the public API from pinned host buffers
        qh = torch.empty(job.q.shape, dtype=torch.float32, pin_memory=True)
        kh = torch.empty(job.k.shape, dtype=torch.float32, pin_memory=True)
        vh = torch.empty(job.v.shape, dtype=torch.float32, pin_memory=True)
        qh.copy_(job.q)
        kh.copy_(job.k)
        vh.copy_(job.v)
        qn, kn, vn = qh.numpy(), kh.numpy(), vh.numpy()
        tables = (job.indptr, job.ids)
        for _ in range(2):
            PagedBatch(job.pool, tables, w.starts, w.n_new).write_and_attend(0, qn, kn, vn)
        e_steps = max(3, min(args.steps, args.e2e_steps))
        ctx.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(ctx.stream)
        for _ in range(e_steps):
            res = PagedBatch(job.pool, tables, w.starts, w.n_new).write_and_attend(0, qn, kn, vn)
        a1.record(ctx.stream)
        ctx.barrier()
        e2e_ms = ctx.max_over_ranks(a0.elapsed_time(a1))
        assert np.isfinite(res).all()

        # the long-context batch over this run's ranks, both layouts
        c5 = {}
        if not args.no_c5:
            steps5 = max(C5_MIN_STEPS, args.steps)
            for layout in ("seq", "head"):
                mk = clocks.mark()
                c5[layout] = measure_c5(ctx, layout, steps5, warmup)
                c5[layout]["clocks"] = clocks.summary(mk)
        configs = {}
        if ctx.world == 1 and not args.no_configs:
            for name in ("c1", "c3", "c4"):
                if name != args.config:
                    mk = clocks.mark()
                    configs[name] = measure_config(ctx, name, max(args.steps, 50), warmup)
                    configs[name]["clocks"] = clocks.summary(mk)

    value = ctx.world * w.rows * args.steps / (ms / 1e3)
    e2e_value = ctx.world * w.rows * e_steps / (e2e_ms / 1e3)
    roof, kind = attention_roofline(
        w, job.batch, prof_ms, prof_n,
        traffic=TC_C2_NCU_TRAFFIC if args.config == "c2" else None)
    if roof["traffic"] is not None:
        roof["traffic_source"] = TC_C2_NCU_SOURCE
    step_bytes = w.algorithmic_bytes()
    uniq = w.unique_kv_bytes()
    result = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": ctx.world,
        "steps": args.steps,
        "warmup": warmup,
        "ms_per_step": round(ms / args.steps, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16" if w.dtype == "bf16" else "f32",
        "data": "synthetic (seeded N(0,1) K/V/q; scattered block tables)",
        "config": {
            "workload": f"{w.name}: {WORKLOAD_TEXT[w.name]}",
            "sequences_per_gpu": w.nseq,
            "rows_per_gpu": w.rows,
            "context_tokens_per_gpu": int(w.ctx_lens.sum()),
            "kv_bytes_per_step_per_gpu": w.kv_read_bytes(),
            "kv_unique_bytes_per_step_per_gpu": uniq,
            "attention_gflop_per_step_per_gpu": round(w.attention_flops() / 1e9, 3),
            "attention_tflops_per_gpu": round(w.attention_flops() / (ms / args.steps / 1e3) / 1e12, 2),
            "cow_pairs_per_step": len(w.cow_pairs),
            "cow_bytes_per_step": w.cow_bytes(),
            "step_algorithmic_bytes_per_gpu": step_bytes,
            "step_gbs_per_gpu": round(step_bytes / (ms / args.steps / 1e3) / 1e9, 1),
            "l2": "inputs larger than L2 (distinct K/V per step > 126 MB)" if uniq > 126e6
                  else "distinct K/V per step fits in L2 (126 MB): L2 flushed (256 MB write) before every timed step",
            "parallelism": f"sequence-sharded x{ctx.world}: the same batch on every GPU, own pool, no collective",
            "job_rows_per_step": ctx.world * w.rows,
            "step": ("copy-on-write copies + " if w.cow_pairs else "")
                    + "append + split-KV attention with in-kernel partial merge, one layer",
        },
        "roofline": roof,
        "e2e": {
            "value": round(e2e_value, 1),
            "unit": "tokens/s",
            "h2d_bytes_per_step": int(job.q.numel() * 4 + job.k.numel() * 8
                                      + (len(job.indptr) * 8 + len(job.ids) * 4) + 16 * w.nseq),
            "d2h_bytes_per_step": int(job.out.numel() * 4),
            "steps": e_steps,
            "path": "PagedBatch(pool, tables, starts, n_new).write_and_attend(0, q, k, v) on pinned numpy; "
                    "the result crosses PCIe as the kernels' stores into the page-locked output",
        },
        "gpu_launches": int(launches_per_step * args.steps),
        "clocks": clk,
    }
    if c5:
        result["c5"] = c5
    if configs:
        result["configs"] = configs
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu:
        tps, dt, reps, threads = cpu_reference(w, args.cpu_seqs, args.cpu_seconds, 200)
        result["cpu_baseline"] = {
            "value": round(tps, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{min(args.cpu_seqs, w.nseq)} of {w.nseq} sequences of the same workload, "
                      f"{reps} steps in {dt:.1f} s (oracle numpy gather path, {cpu_model()}, "
                      f"{os.cpu_count()} logical CPUs)",
        }
    if ctx.rank == 0:
        print(json.dumps(result), file=RESULT_OUT, flush=True)
    job.close()
    if ctx.world > 1:
        ctx.dist.barrier()
        ctx.dist.destroy_process_group()


# ------------------------------------------------------------------------------ reference arm
def _pagellm():
    """pagellm's own cache module from the offline install in baseline/_ref, or None."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "pagellm").is_dir():
        return None
    sys.path.insert(0, str(ref))
    try:
        from pagellm.cache import paged  # noqa: PLC0415

        return paged
    except Exception:  # noqa: BLE001 - an unusable install falls back to the port
        return None
    finally:
        sys.path.remove(str(ref))


def run_reference(args):
    """pagellm's numpy path on this host's cores (rank 0 only): the unmodified
    ``PagedBatch(pool, tables, starts, n_new, "gather").write_and_attend`` from the install in
    baseline/_ref on the whole workload, timed at all host threads (the line's value) and at
    pagellm's default of one BLAS thread (pagellm/__init__.py sets it before numpy loads)."""
    from threadpoolctl import threadpool_limits

    from pagellm_b200 import workloads

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = workloads.make(args.config, seed=0)
    paged = _pagellm()
    x = cpu_inputs(w, list(range(w.nseq)), 0)
    cores = os.cpu_count() or 1
    if paged is not None:
        class Shape:
            n_layers, n_kv_heads, head_dim = 1, w.KVH, w.D

        pool = paged.PagedKVPool(Shape, x["nb"], w.bs, np.float32)
        pool.k_flat[0][:] = x["kp"]
        pool.v_flat[0][:] = x["vp"]

        def step():
            for src, dst in x["pairs"]:  # the step's copy-on-write copies, as LLMEngine.step makes them
                pool.copy_block(src, dst)
            return paged.PagedBatch(pool, x["tables"], x["starts"], x["n_new"], "gather").write_and_attend(
                0, x["q"], x["k"], x["v"])

        kind, what = "reference", "pagellm PagedBatch(..., 'gather').write_and_attend from baseline/_ref"
    else:
        from oracle import paged_oracle as po

        def step():
            blk = (1, x["nb"], w.bs, w.KVH, w.D)
            po.copy_blocks(x["kp"].reshape(blk), x["vp"].reshape(blk), x["pairs"])
            meta = po.StepMeta(x["tables"], x["starts"], x["n_new"], w.bs)
            return po.write_and_attend(x["kp"], x["vp"], meta, x["q"], x["k"], x["v"])

        kind, what = "port", "oracle/paged_oracle.py numpy port (baseline/_ref not importable)"

    def timed(threads: int, steps: int, warmup: int, budget_s: float):
        with threadpool_limits(limits=threads):
            for _ in range(warmup):
                step()
            t0 = time.perf_counter()
            n = 0
            while n < steps and (n == 0 or time.perf_counter() - t0 < budget_s):
                step()
                n += 1
            return n, time.perf_counter() - t0

    warm = max(args.warmup, 1)
    # all host threads: the line's value; K steps unless that would run past the budget
    n_all, dt_all = timed(cores, args.steps, min(warm, 2), args.ref_seconds)
    # pagellm's own default (one BLAS thread), a shorter sample
    n_one, dt_one = timed(1, max(1, min(args.steps, 3)), 1, args.ref_seconds / 3)
    tps = w.rows * n_all / dt_all
    tps1 = w.rows * n_one / dt_one
    sample = (f"all {w.nseq} sequences of the workload per step ({w.rows} rows, "
              f"{int(w.ctx_lens.sum())} context tokens), {n_all} timed steps of {args.steps} requested "
              f"in {dt_all:.1f} s ({cpu_model()}, {cores} logical CPUs)")
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC,
        "value": round(tps, 3),
        "unit": "tokens/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": n_all,
        "steps_requested": args.steps,
        "warmup": min(warm, 2),
        "ms_per_step": round(dt_all / n_all * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1); bf16-rounded K/V for bf16 workloads)",
        "config": {"workload": f"{w.name}: {WORKLOAD_TEXT[w.name]}", "sequences_per_step": w.nseq,
                   "rows_per_step": w.rows, "path": what},
        "cpu_baseline": {"value": round(tps, 3), "unit": "tokens/s", "cores": cores, "kind": kind,
                         "sample": sample},
        "one_blas_thread": {"value": round(tps1, 3), "unit": "tokens/s", "cores": 1, "steps": n_one,
                            "ms_per_step": round(dt_one / n_one * 1e3, 3),
                            "note": "pagellm's default (OPENBLAS/OMP/MKL threads = 1)"},
        "e2e": {"value": round(tps, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), file=RESULT_OUT, flush=True)


def _claim_stdout():
    """Keep stdout for the one JSON line: libraries (NCCL prints a version banner) write
    through file descriptor 1, which is pointed at stderr for the rest of the run."""
    out = os.fdopen(os.dup(1), "w", buffering=1)
    sys.stdout.flush()
    os.dup2(2, 1)
    return out


def main():
    global RESULT_OUT
    RESULT_OUT = _claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=100)
    ap.add_argument("--cpu-seqs", type=int, default=8)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--ref-seconds", type=float, default=90.0,
                    help="reference arm: time budget of its all-thread steps")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-c5", action="store_true")
    ap.add_argument("--no-configs", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
