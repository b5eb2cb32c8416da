"""Benchmark: one AB-attention layer (fresh plan + HT sparse prefill) at the
Wan2.1-14B 720p shape (B=2, H=40, 75,600 tokens, 64 sampled pages), heads
sharded over N B200 GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config wan14b] [--impl ours|reference]

A step is `build_plan` + `apply_plan` over the whole layer (on N > 1 each rank
does its contiguous head shard, then one NCCL all-gather reassembles the
output). Rank 0 prints one JSON line; `value` is the whole-job layer time in ms
(max over ranks, CUDA events, inputs resident in HBM; the inputs are larger
than L2, so no flush is needed between steps). `e2e` repeats the measurement
through the public API with the step's inputs copied from pinned host memory
and the output copied back inside the timed region.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "AB-attn layer ms + eff. TFLOP/s at Wan2.1-14B 720p shape, 1/2/4/8 B200"


# ---- helpers -------------------------------------------------------------------

def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16_tflops": data["bf16_tflops"],
                "bf16_tflops_sustained": data.get("bf16_tflops_sustained", data["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons every 20 ms. It is started
    before the warm-up (nvidia-smi takes a moment to start) and keeps only the
    samples that arrive inside the timed window (`mark_start` .. `mark_stop`)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self.window = (0.0, float("inf"))

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def mark_start(self):
        self.window = (time.monotonic(), float("inf"))

    def mark_stop(self):
        self.window = (self.window[0], time.monotonic() + 0.025)  # a sample in flight at the end

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        lo, hi = self.window
        for when, line in self.lines:
            if not lo <= when <= hi:
                continue
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# DRAM bytes (read + write) of one paired prefill launch per head at the Wan shape,
# from one ncu capture of the 2-head case (dram__bytes_read.sum + dram__bytes_write.sum
# = 138.85 + 21.98 MB); a head's K/V stay L2-resident, so traffic scales with heads.
PREFILL_DRAM_BYTES_PER_HEAD = (138.85e6 + 21.98e6) / 2


def plan_bytes(bh: int, tokens: int, samples: int) -> float:
    """Algorithmic HBM bytes of build_plan: read Q and K once, write ids + weights."""
    rows = bh * math.ceil(tokens / 128)
    return 2.0 * bh * tokens * 128 * 2 + rows * samples * 8


def layer_flops(bh: int, tokens: int, keys_per_row: int) -> float:
    """4*D*BH*S*keys: QK^T and PV of the sparse prefill (D = 128)."""
    return 4.0 * 128 * bh * tokens * keys_per_row


def dense_flops(bh: int, tokens: int) -> float:
    return 4.0 * 128 * bh * tokens * tokens


# ---- CPU baseline (the oracle port, bounded sample) -----------------------------

def _cpu_rows(task) -> tuple[float, float]:
    """Worker: the CPU restatement of the layer (IBCS + SIP + prefill) on
    `count` query blocks of one head; returns (pool seconds, rows seconds)."""
    name, frames, height, width, seed, samples, first, count = task
    import numpy as np
    from threadpoolctl import threadpool_limits

    sys.path.insert(0, str(ROOT))
    from ab_attention_b200.synthetic import smooth_field
    from oracle import oracle

    with threadpool_limits(1):
        q, k, v = smooth_field(1, frames, height, width, seed=seed, device="cpu")
        bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        # per-head work: key pooling and the float64 copies of K and V
        t0 = time.perf_counter()
        pooled = oracle.pool(bits(k))
        k64, v64 = k.double().numpy(), v.double().numpy()
        t_pool = time.perf_counter() - t0
        sub = bits(q)[:, first * 128:(first + count) * 128]
        q64 = q[:, first * 128:(first + count) * 128].double().numpy()
        # per-row work: clustering, centroid scores, mixture, SIP, sparse prefill
        t0 = time.perf_counter()
        cent, pops, _ = oracle.cluster(sub)
        lse, mx, den = oracle.lse(cent, pooled, 1, count)
        scores = oracle.mix(lse, pops, mx, den)
        ids, logw = oracle.sip(scores, np.full(count, 0.5, np.float32), samples)
        oracle.prefill(q64, k64, v64, ids, logw)
        t_rows = time.perf_counter() - t0
    return t_pool, t_rows


def cpu_sample(shape, rows_per_worker: int = 24, workers: int = 1, pool=None) -> dict:
    """Time the CPU restatement on a bounded sample (rows_per_worker query blocks
    per worker process, plus one head's key pooling per worker) and extrapolate
    linearly to the whole layer. Returns ms per layer. `pool`: an existing
    process pool with `workers` processes (else one is started for the call)."""
    qb = math.ceil(shape.tokens / 128)
    rows_total = shape.batch_heads * qb
    tasks = [(shape.name, shape.frames, shape.height, shape.width, shape.seed, shape.sample_pages * 32,
              (w * rows_per_worker) % max(1, qb - rows_per_worker), rows_per_worker) for w in range(workers)]
    t0 = time.perf_counter()
    if workers == 1:
        results = [_cpu_rows(tasks[0])]
    elif pool is not None:
        results = list(pool.map(_cpu_rows, tasks))
    else:
        import concurrent.futures as cf
        import multiprocessing as mp

        with cf.ProcessPoolExecutor(max_workers=workers, mp_context=mp.get_context("spawn")) as pool:
            results = list(pool.map(_cpu_rows, tasks))
    wall = time.perf_counter() - t0
    t_pool = statistics.mean(r[0] for r in results)
    t_rows = statistics.mean(r[1] for r in results)
    # each worker handles its own rows in parallel: rows/s = workers * rows_per_worker / t_rows
    ms = (rows_total * t_rows / (workers * rows_per_worker) + shape.batch_heads * t_pool / workers) * 1e3
    return {"value": ms, "unit": "ms", "cores": workers,
            "sample": f"{rows_per_worker} query blocks of one head per worker x {workers} worker(s) "
                      f"(C oracle: IBCS + SIP; float64 numpy prefill) + that head's key pooling, "
                      f"extrapolated linearly to {rows_total} blocks / {shape.batch_heads} heads",
            "sample_seconds": wall}


def run_reference(args, shape) -> None:
    """`--impl reference`: the reference's math on the host cores. The reference
    has no CPU implementation of its own (its kernels are CUDA), so this arm
    runs the CPU restatement in oracle/ with one worker process per core."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import concurrent.futures as cf
    import multiprocessing as mp

    cores = os.cpu_count() or 1
    rows_per_worker = 24  # ~50 ms of CPU per query block: about 1 s per worker per step
    with cf.ProcessPoolExecutor(max_workers=cores, mp_context=mp.get_context("spawn")) as pool:
        for _ in range(args.warmup):
            cpu_sample(shape, rows_per_worker=2, workers=cores, pool=pool)
        values = [cpu_sample(shape, rows_per_worker=rows_per_worker, workers=cores, pool=pool)["value"]
                  for _ in range(args.steps)]
    value = statistics.median(values)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "ms", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": value, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic smooth-field video tokens",
        "config": {"workload": shape.name, "batch": shape.batch, "heads": shape.heads, "tokens": shape.tokens,
                   "sample_pages": shape.sample_pages},
        "cpu_baseline": {"value": value, "unit": "ms", "cores": cores, "kind": "port",
                         "sample": f"{rows_per_worker} query blocks of one head per worker x {cores} workers per step "
                                   f"(C/numpy restatement of the reference math), extrapolated to the layer"},
        "e2e": {"value": value, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- GPU arm -----------------------------------------------------------------------

def phase_times_sharded(abx, shard, q, k, v, offsets, gathered, world, chunks, shape, text, stream, reps=3):
    """Median (plan ms, prefill + overlapped all-gather ms) of a sharded step,
    timed as two halves: build_plan alone, then the whole step minus it."""
    import torch.distributed as dist

    plans, totals = [], []
    for _ in range(reps):
        dist.barrier()
        a, b, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record(stream)
        abx.build_plan(q, k, sample_pages=shape.sample_pages, offsets=offsets)
        b.record(stream)
        shard.attention_sharded(q, k, v, offsets, gathered, world=world, chunks=chunks,
                                sample_pages=shape.sample_pages, text_kv=text)
        c.record(stream)
        torch.cuda.synchronize()
        plans.append(a.elapsed_time(b))
        totals.append(b.elapsed_time(c))
    plan = statistics.median(plans)
    return plan, max(0.0, statistics.median(totals) - plan)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--config", default="wan14b")
    parser.add_argument("--impl", default="ours", choices=["ours", "reference"])
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-dense", action="store_true")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--sample-pages", type=int, default=0,
                        help="override the configuration's sampled pages per row (the C4 sweep: 16..256)")
    parser.add_argument("--bh", type=int, default=0,
                        help="run only the first BH (batch*head) rows of the configuration (profiling)")
    args = parser.parse_args()

    from ab_attention_b200.synthetic import CONFIGS, make_inputs

    shape = CONFIGS[args.config]
    if args.sample_pages:
        import dataclasses

        shape = dataclasses.replace(shape, name=f"{shape.name}[p={args.sample_pages}]", sample_pages=args.sample_pages)
    if args.bh:
        import dataclasses

        shape = dataclasses.replace(shape, name=f"{shape.name}[bh={args.bh}]", batch=1, heads=args.bh)
    if args.impl == "reference":
        run_reference(args, shape)
        return

    import ab_attention_b200 as abx
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        # NCCL prints its version banner on stdout while it creates the communicator;
        # route it to stderr so that rank 0's stdout carries only the JSON line.
        sys.stdout.flush()
        saved_stdout = os.dup(1)
        try:
            os.dup2(2, 1)
            dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
            dist.barrier(device_ids=[local])
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)
    from ab_attention_b200 import shard

    bh = shape.batch_heads
    chunks = shard.chunk_count(bh, world) if world > 1 else 1
    heads = shard.rank_heads(bh, world, rank, chunks)
    per = len(heads)
    q, k, v, text = make_inputs(shape, device=device, bh_slice=heads if world > 1 else None)
    q, k, v = (x.reshape(1, per, shape.tokens, 128).contiguous() for x in (q, k, v))
    if text is not None:
        text = tuple(t.reshape(1, per, -1, 128).contiguous() for t in text)
    tokens = shape.tokens
    offsets = shard.shard_offsets(shard.layer_offsets(bh, tokens, shape.seed, device), tokens, heads)
    gathered = torch.empty((bh, tokens, 128), dtype=torch.bfloat16, device=device) if world > 1 else None

    def barrier():
        if world > 1:
            dist.barrier()

    stream = torch.cuda.current_stream(device)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]

    def step(i=None, qq=q, kk=k, vv=v):
        e = ev[i] if i is not None else None
        if world > 1:
            # plan for all local heads, prefill by head block, each block's
            # all-gather overlapping the next block's prefill
            if e:
                e[0].record(stream)
            shard.attention_sharded(qq, kk, vv, offsets, gathered, world=world, chunks=chunks,
                                    sample_pages=shape.sample_pages, text_kv=text)
            if e:
                e[1].record(stream)
            return gathered
        if e:
            e[0].record(stream)
        plan = abx.build_plan(qq, kk, sample_pages=shape.sample_pages, offsets=offsets)
        if e:
            e[1].record(stream)
        o = abx.apply_plan(qq, kk, vv, plan, text_kv=text)
        if e:
            e[2].record(stream)
        return o

    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        for _ in range(max(3, args.warmup)):
            step()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        clocks.mark_start()
        start.record(stream)
        for i in range(args.steps):
            step(i)
        stop.record(stream)
        torch.cuda.synchronize()
        clocks.mark_stop()
    barrier()
    elapsed = start.elapsed_time(stop)
    if world > 1:
        # phases of one step measured separately (untimed for the headline): plan,
        # then prefill + overlapped all-gathers
        plan_ms, prefill_ms = phase_times_sharded(abx, shard, q, k, v, offsets, gathered, world, chunks, shape,
                                                  text, stream)
    else:
        plan_ms = statistics.median(e[0].elapsed_time(e[1]) for e in ev)
        prefill_ms = statistics.median(e[1].elapsed_time(e[2]) for e in ev)
    t = torch.tensor([elapsed, plan_ms, prefill_ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed, plan_ms, prefill_ms = t.tolist()
    ms = elapsed / args.steps

    # End to end through the public API: pinned host inputs in, output back out.
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
        hout = torch.empty(q.shape, dtype=q.dtype).pin_memory()
        h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv))
        d2h = hout.numel() * hout.element_size()

        def e2e_step():
            # head blocks stream through: block c + 1 copied in while block c is
            # planned, attended and all-gathered, block c's own heads copied out
            return shard.attention_sharded_host(hq, hk, hv, offsets, gathered, hout, world=world, chunks=chunks,
                                                sample_pages=shape.sample_pages, text_kv=text)

        if world == 1:
            # the public host-buffer entry point: copy-in, compute and copy-out of
            # head chunks overlap on three streams (prompt keys stay on the device)
            def e2e_step():  # noqa: F811
                return abx.ab_attention_host(hq, hk, hv, sample_pages=shape.sample_pages, seed=shape.seed,
                                             out=hout.view(q.shape), device=device, text_kv=text)

        e2e_step()
        torch.cuda.synchronize()
        barrier()
        s2, t2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2e_steps = max(2, min(args.steps, 5))
        s2.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        t2.record(stream)
        torch.cuda.synchronize()
        tt = torch.tensor([s2.elapsed_time(t2) / e2e_steps], device=device)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e = {"value": tt.item(), "unit": "ms", "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world}
        del hq, hk, hv, hout

    # Dense comparators (1 GPU only): this build's prefill in dense mode and cuDNN SDPA.
    dense = {}
    if world == 1 and not args.no_dense:
        def timed(fn, reps=2):
            fn()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(reps):
                fn()
            b.record(stream)
            torch.cuda.synchronize()
            return a.elapsed_time(b) / reps

        dense["own_dense_ms"] = timed(lambda: abx.dense_attention(q, k, v))
        try:
            from torch.nn.attention import SDPBackend, sdpa_kernel

            with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
                dense["cudnn_sdpa_ms"] = timed(
                    lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v))
        except Exception as exc:  # noqa: BLE001
            dense["cudnn_sdpa_error"] = str(exc)[:200]
        best = min(v_ for k_, v_ in dense.items() if k_.endswith("_ms"))
        dense["dense_ms"] = best
        dense["speedup_vs_dense"] = best / ms

    keys_per_row = shape.sample_pages * 128 + shape.text_tokens
    sparse_flops = layer_flops(bh, tokens, keys_per_row)
    eq_flops = dense_flops(bh, tokens)
    peaks = measured_peaks()
    prefill_flops_rank = layer_flops(per, tokens, keys_per_row)
    achieved = prefill_flops_rank / (prefill_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": ms, "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic smooth-field video tokens (seeded), random per-head projections",
        "config": {"workload": shape.name, "batch": shape.batch, "heads": shape.heads, "tokens": tokens,
                   "grid": [shape.frames, shape.height, shape.width], "sample_pages": shape.sample_pages,
                   "text_tokens": shape.text_tokens, "parallelism": f"heads{world}",
                   "l2": "inputs (Q/K/V 4.6 GB) larger than L2; no flush",
                   "step": "build_plan (fresh plan) + apply_plan"
                           + (f" in {chunks} head blocks, each all-gathered while the next computes"
                              if world > 1 else "")},
        "eff_tflops": eq_flops / (ms * 1e-3) / 1e12,
        "sparse_tflops": sparse_flops / (ms * 1e-3) / 1e12,
        "plan_ms": plan_ms, "prefill_ms": prefill_ms,
        "plan_amortised_ms": prefill_ms + plan_ms / 4,
        "roofline": {"kernel": "sparse prefill", "bound": "tensor", "achieved": achieved,
                     "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops_sustained"],
                     # the per-head figure was captured at the wan14b shape with 64 pages
                     "traffic": (PREFILL_DRAM_BYTES_PER_HEAD * per
                                 if shape.name.split("[")[0] == "wan14b" and shape.sample_pages == 64 else None),
                     "peak_source": peaks["source"] + " sustained bf16"},
        "plan_roofline": {"kernels": "cluster (with the key pooling) + lse + sip (mixture evaluated inside sip)", "bound": "hbm",
                          "achieved": plan_bytes(per, tokens, shape.sample_pages * 32) / (plan_ms * 1e-3) / 1e9,
                          "peak": peaks["hbm_gbs"], "unit": "GB/s",
                          "frac": plan_bytes(per, tokens, shape.sample_pages * 32) / (plan_ms * 1e-3) / 1e9
                          / peaks["hbm_gbs"],
                          "note": "algorithmic bytes (Q, K in; plan out); the kernels are bound by the exact "
                                  "fast-math exp2/log2/division work and the double-precision SIP sums"},
        # cluster, pool, lse, sip + a pair plan and a prefill per head block per step
        # (NCCL's kernels not counted)
        "gpu_launches": (3 + 2 * chunks) * args.steps,
        "clocks": clocks.summary(),
        **dense,
    }
    if e2e is not None:
        line["e2e"] = e2e
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_sample(shape, rows_per_worker=192, workers=1)  # ~10 s of one core
        line["cpu_baseline"]["kind"] = "port"
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
