"""Benchmark of the paged KV-cache hot path on B200: decode-attention tokens/s and HBM GB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

One step = one layer of ``PagedBatch.write_and_attend`` for the workload (append the new
K/V rows through the slot mapping, then split-KV GQA attention over the paged cache) on
seeded synthetic inputs; default workload C2 (Llama-3-8B shape, batch 64, bf16 K/V,
contexts U{512..4096}). Under torchrun every rank runs its own batch on its own pool
(sequence-sharded, no collective on the data path): weak scaling.

* ``value``: tokens/s over all ranks, K steps timed with CUDA events (inputs resident).
* ``e2e``: the same through the public Python API from pinned HOST buffers, every step
  re-planning the batch (block tables up), q/k/v up and the output down.
* ``roofline``: the dominant kernel's algorithmic bytes (split-KV decode) or FLOPs (the
  tcgen05 wide-tile pass, C3/C4) per event-timed launch against the measured HBM copy
  bandwidth or sustained bf16 throughput (MEASURED_PEAKS.json).
* ``cpu_baseline``: the CPU oracle (numpy restatement of pagellm's gather path) on a
  bounded sample of the same workload on this host.
``--impl reference`` times that CPU path alone (rank 0; other ranks exit).
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
TC_C2_NCU_TRAFFIC = 625_797_376  # dram__bytes_read.sum + dram__bytes_write.sum, one C2 launch
RESULT_OUT = sys.stdout


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

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in self.rows if num(r[1])]
        mx = [num(r[2]) for r in self.rows if num(r[2])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ------------------------------------------------------------------------------ CPU path
def cpu_reference(w, sample_seqs: int, min_seconds: float, max_reps: int, seed: int = 0):
    """The oracle's numpy port of pagellm's gather path (append + padded batched decode)
    on ``sample_seqs`` sequences of workload ``w``; K/V bf16-rounded for bf16 workloads.
    Returns (tokens/s, seconds, reps, threads)."""
    from oracle import paged_oracle as po

    rng = np.random.default_rng(seed)
    sel = list(range(min(sample_seqs, w.nseq)))
    bs, kvh, d = w.bs, w.KVH, w.D
    # compact host pool holding only the sampled sequences' blocks
    tables, nb = [], 0
    for i in sel:
        n = len(w.tables[i])
        tables.append(list(range(nb, nb + n)))
        nb += n
    kp = rng.standard_normal((nb * bs, kvh, d), dtype=np.float32)
    vp = rng.standard_normal((nb * bs, kvh, d), dtype=np.float32)
    if w.dtype == "bf16":
        kp, vp = po.bf16_round(kp), po.bf16_round(vp)
    starts = [int(w.starts[i]) for i in sel]
    n_new = [int(w.n_new[i]) for i in sel]
    rows = sum(n_new)
    q = rng.standard_normal((rows, w.H, d), dtype=np.float32)
    k = rng.standard_normal((rows, kvh, d), dtype=np.float32)
    v = rng.standard_normal((rows, kvh, d), dtype=np.float32)
    if w.dtype == "bf16":
        k, v = po.bf16_round(k), po.bf16_round(v)
    meta = po.StepMeta(tables, starts, n_new, bs)
    po.write_and_attend(kp, vp, meta, q, k, v)  # warm-up
    t0 = time.perf_counter()
    reps = 0
    while reps < max_reps and (reps == 0 or time.perf_counter() - t0 < min_seconds):
        meta = po.StepMeta(tables, starts, n_new, bs)
        po.write_and_attend(kp, vp, meta, q, k, v)
        reps += 1
    dt = time.perf_counter() - t0
    threads = int(os.environ.get("OPENBLAS_NUM_THREADS") or os.environ.get("OMP_NUM_THREADS") or os.cpu_count())
    return rows * reps / dt, dt, reps, threads


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ------------------------------------------------------------------------------ GPU path
def run_ours(args):
    import torch
    import torch.distributed as dist

    from pagellm_b200 import _lib, workloads
    from pagellm_b200.cache import PagedBatch, PagedKVPool

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from pagellm_b200.sharding import gather_heads, shard_sequences

    head_mode = args.config == "c5" and args.shard == "head"
    if args.config == "c5":
        # one fixed batch of 128 sequences split over the ranks: strong scaling
        L = workloads.c5_lengths(0)
        if head_mode:
            w = workloads.c5(0, lengths=L, kv_heads=8 // world)
        else:
            w = workloads.c5(0, lengths=L[shard_sequences(L, world)[rank]])
        scaling, total_rows = "strong", len(L)
    else:
        w = workloads.make(args.config, seed=rank)
        scaling, total_rows = "weak", None

    class Shape:
        n_layers, n_kv_heads, head_dim = 1, w.KVH, w.D

    pool = PagedKVPool(Shape, w.num_blocks, w.bs, "bfloat16" if w.dtype == "bf16" else np.float32)
    g = torch.Generator(device=dev).manual_seed(rank)
    for t in (pool.k, pool.v):
        t[0].copy_(torch.randn(t[0].shape, generator=g, device=dev).to(t.dtype))
    pairs_dev = None
    if w.cow_pairs:
        pairs_dev = torch.as_tensor(np.asarray(w.cow_pairs, dtype=np.int64).reshape(-1, 2), device=dev)
        pool.copy_blocks(w.cow_pairs)
    indptr, ids = w.csr()
    batch = PagedBatch(pool, (indptr, ids), w.starts, w.n_new)
    q = torch.randn((w.rows, w.H, w.D), generator=g, device=dev)
    k = torch.randn((w.rows, w.KVH, w.D), generator=g, device=dev)
    v = torch.randn((w.rows, w.KVH, w.D), generator=g, device=dev)
    out = torch.empty_like(q)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev)
    st = stream.cuda_stream

    def step():
        if head_mode:
            attend_layer()
            if world > 1:  # one rank holds every head: nothing to gather
                gather_heads(out)
            return
        if pairs_dev is not None:  # the step's copy-on-write copies (fork of the shared block)
            rc = lib.pk_pool_copy_blocks_dev(pool.handle, pairs_dev.data_ptr(), len(pairs_dev), st)
            if rc:
                _lib.check(rc)
        rc = lib.pk_batch_write_and_attend(batch._b, 0, w.H, q.data_ptr(), k.data_ptr(),
                                           v.data_ptr(), out.data_ptr(), st)
        if rc:
            _lib.check(rc)

    def attend_layer():
        rc = lib.pk_batch_write_and_attend(batch._b, 0, w.H, q.data_ptr(), k.data_ptr(),
                                           v.data_ptr(), out.data_ptr(), st)
        if rc:
            _lib.check(rc)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with ClockSampler(local) as clocks:
        for _ in range(max(args.warmup, 3)):
            step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1))
        batch.check()
        launches_per_step = batch.stats()["launches"] + (1 if pairs_dev is not None else 0)

        # kernel timing for the roofline (events on the launching stream, same K steps)
        lib.pk_batch_profile(batch._b, 1)
        for _ in range(args.steps):
            (attend_layer if head_mode else step)()
        prof_ms = (C.c_double * 5)()
        prof_n = (C.c_int64 * 5)()
        _lib.check(lib.pk_batch_profile_read(batch._b, prof_ms, prof_n))
        lib.pk_batch_profile(batch._b, 0)
        barrier()

        # end to end through the public API from pinned host buffers
        qh = torch.empty(q.shape, dtype=torch.float32, pin_memory=True)
        kh = torch.empty(k.shape, dtype=torch.float32, pin_memory=True)
        vh = torch.empty(v.shape, dtype=torch.float32, pin_memory=True)
        qh.copy_(q)
        kh.copy_(k)
        vh.copy_(v)
        qn, kn, vn = qh.numpy(), kh.numpy(), vh.numpy()
        for _ in range(2):
            PagedBatch(pool, (indptr, ids), w.starts, w.n_new).write_and_attend(0, qn, kn, vn)
        e_steps = max(3, min(args.steps, args.e2e_steps))
        barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(e_steps):
            res = PagedBatch(pool, (indptr, ids), w.starts, w.n_new).write_and_attend(0, qn, kn, vn)
            if head_mode and world > 1:  # slices back to the GPU, all-gather, full output to the host
                res = gather_heads(torch.from_numpy(res).to(dev)).cpu().numpy()
        a1.record(stream)
        barrier()
        e2e_ms = max_over_ranks(a0.elapsed_time(a1))
        assert np.isfinite(res).all()
    clk = clocks.summary()

    job_rows = total_rows if total_rows is not None else world * w.rows
    value = job_rows * args.steps / (ms / 1e3)
    e2e_value = job_rows * e_steps / (e2e_ms / 1e3)
    hbm, hbm_src = peaks()
    # dominant kernel: tensor-core split-KV attention (kind 1); algorithmic bytes per launch:
    # the distinct K/V blocks it must read (shared blocks once), q in, out, tables, metadata
    uniq = w.unique_kv_bytes()
    alg_attn = (uniq + w.rows * w.H * w.D * 8
                + int(sum(-(-int(L) // w.bs) for L in w.ctx_lens)) * 4 + w.nseq * 12)
    # the dominant attention kernel of this workload (most total time)
    kind = max((1, 3, 4), key=lambda i: prof_ms[i])
    avg_ms = prof_ms[kind] / max(1, prof_n[kind])
    achieved = alg_attn / (avg_ms / 1e3) / 1e9
    # the tcgen05 kernel's algorithmic FLOPs (Q.K^T + P.V over the keys each row sees): the
    # causal chunks it takes (>= 64 query rows per KV head) plus the shared-prefix pass
    g = w.H // w.KVH
    chunk_tk = sum(sum(int(w.starts[i]) + t + 1 for t in range(int(w.n_new[i])))
                   for i in range(w.nseq) if int(w.n_new[i]) * g >= 64)
    wide_flops = 4.0 * w.H * w.D * (chunk_tk + batch.prefix_stats()["token_keys"])
    step_bytes = w.algorithmic_bytes()
    result = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms / args.steps, 5),
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": "bf16" if w.dtype == "bf16" else "f32",
        "data": "synthetic (seeded N(0,1) K/V/q; scattered block tables)",
        "config": {
            "workload": f"{w.name}: " + {
                "c1": "fp32 decode B=8 H=4 KVH=2 d=32 bs=16 L~U{1..256}",
                "c2": "Llama-3-8B decode attention, 1 layer, B=64 H=32 KVH=8 d=128 bs=16, L~U{512..4096}, bf16 K/V fp32 accumulate",
                "c3": "mixed step: 16 decodes L~U{256..2048} + 512-query chunk at 1024..1535",
                "c4": "64 requests x 4 forks share a 2048-token prefix, 192 CoW copies, 5-token verify",
                "c5": "70B long-context decode B=128 H=64 KVH=8 d=128, L~lognormal(8192,0.75) clip[1024,32768]",
            }[w.name],
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
                  else "distinct K/V per step fits in L2 (126 MB): not flushed, achieved GB/s counts distinct bytes",
            "parallelism": (f"head-sharded x{world}: {w.KVH} KV heads per GPU for all sequences, "
                            "NCCL all-gather of the output slices inside the step") if head_mode else
                           (f"sequence-sharded x{world} (own pool per GPU, no collective)"
                            + (", 128-sequence batch split longest-first" if args.config == "c5" else "")),
            "job_rows_per_step": job_rows,
            "step": ("copy-on-write copies + " if w.cow_pairs else "")
                    + "append + split-KV attention with in-kernel partial merge, one layer",
        },
        "roofline": {
            "bound": "hbm",
            "kernel": {1: "tc_attn_kernel (split-KV paged attention, TMA + mma.sync bf16)",
                       3: "generic_attn_kernel (CUDA cores)",
                       4: "wide_attn_kernel (tcgen05/TMEM chunk attention, TMA)"}[kind],
            "achieved": round(achieved, 1),
            "peak": hbm,
            "unit": "GB/s",
            "frac": round(achieved / hbm, 4),
            "peak_source": hbm_src,
            # DRAM read + write bytes of one launch from ncu (profiles/tc_attn_kernel_c2.md);
            # recorded for the default workload only
            "traffic": TC_C2_NCU_TRAFFIC if (args.config == "c2" and world == 1 and kind == 1) else None,
            "algorithmic_bytes_per_launch": alg_attn,
            "avg_launch_us": round(avg_ms * 1e3, 2),
            "kernel_us": {n: round(prof_ms[i] / max(1, prof_n[i]) * 1e3, 2)
                          for i, n in enumerate(("append", "tc_attention", "merge", "cuda_core_attention",
                                                 "wide_tcgen05_attention"))
                          if prof_n[i]},
        },
        "e2e": {
            "value": round(e2e_value, 1),
            "unit": "tokens/s",
            "h2d_bytes_per_step": int(q.numel() * 4 + k.numel() * 8 + (len(indptr) * 8 + len(ids) * 4)
                                      + 16 * w.nseq),
            "d2h_bytes_per_step": int(out.numel() * 4),
            "steps": e_steps,
            "path": "PagedBatch(pool, tables, starts, n_new).write_and_attend(0, q, k, v) on pinned numpy; "
                    "the result crosses PCIe as the kernels' stores into the page-locked output",
        },
        "gpu_launches": int(launches_per_step * args.steps),
        "clocks": clk,
    }
    if kind == 4:
        # compute-bound wide-tile pass: report it against the tensor roofline
        tp, tp_src = tensor_peak()
        tflops = wide_flops / (avg_ms / 1e3) / 1e12
        result["roofline"].update({
            "bound": "tensor", "achieved": round(tflops, 1), "peak": tp, "unit": "TFLOP/s",
            "frac": round(tflops / tp, 4), "peak_source": tp_src,
            "algorithmic_flops_per_launch": wide_flops, "algorithmic_bytes_per_launch": None,
        })
    if rank == 0 and world == 1 and not args.no_cpu:
        tps, dt, reps, threads = cpu_reference(w, args.cpu_seqs, args.cpu_seconds, 200)
        result["cpu_baseline"] = {
            "value": round(tps, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{min(args.cpu_seqs, w.nseq)} of {w.nseq} sequences of the same workload, "
                      f"{reps} steps in {dt:.1f} s (oracle numpy gather path, {cpu_model()}, "
                      f"{os.cpu_count()} logical CPUs)",
        }
    if rank == 0:
        print(json.dumps(result), file=RESULT_OUT, flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args):
    """The reference's CPU algorithm (oracle port of pagellm's numpy path), rank 0 only."""
    from pagellm_b200 import workloads

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = workloads.make(args.config, seed=0)
    for _ in range(max(args.warmup, 1)):
        cpu_reference(w, args.cpu_seqs, 0.0, 1)
    tps, dt, reps, threads = cpu_reference(w, args.cpu_seqs, 0.0, args.steps)
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC,
        "value": round(tps, 2),
        "unit": "tokens/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps,
        "warmup": max(args.warmup, 1),
        "ms_per_step": round(dt / reps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1); bf16-rounded K/V for bf16 workloads)",
        "config": {"workload": w.name, "sequences_per_step": min(args.cpu_seqs, w.nseq),
                   "note": "CPU numpy port of pagellm's PagedBatch gather path (oracle/paged_oracle.py)"},
        "cpu_baseline": {"value": round(tps, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{min(args.cpu_seqs, w.nseq)} of {w.nseq} sequences per step, "
                                   f"{reps} steps ({cpu_model()}, {os.cpu_count()} logical CPUs)"},
        "e2e": {"value": round(tps, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
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
    ap.add_argument("--shard", default="seq", choices=["seq", "head"],
                    help="c5 multi-GPU layout: whole sequences per GPU, or KV heads per GPU + all-gather")
    ap.add_argument("--e2e-steps", type=int, default=100)
    ap.add_argument("--cpu-seqs", type=int, default=8)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
