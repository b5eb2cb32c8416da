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
    """Samples nvidia-smi SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

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
        for line in self.lines:
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


def layer_flops(bh: int, tokens: int, keys_per_row: int) -> float:
    """4*D*BH*S*keys: QK^T and PV of the sparse prefill (D = 128)."""
    return 4.0 * 128 * bh * tokens * keys_per_row


def dense_flops(bh: int, tokens: int) -> float:
    return 4.0 * 128 * bh * tokens * tokens


# ---- CPU baseline (the oracle port, bounded sample) -----------------------------

def cpu_sample(shape, rows_sample: int = 8, threads: int = 1) -> dict:
    """Time the CPU restatement of the layer on `rows_sample` query blocks of one
    head (IBCS + SIP + prefill) plus the per-head key pooling, and extrapolate
    linearly to the whole layer. Returns ms per layer."""
    import numpy as np
    from threadpoolctl import threadpool_limits

    from ab_attention_b200.synthetic import smooth_field
    from oracle import oracle

    q, k, v = smooth_field(1, shape.frames, shape.height, shape.width, seed=shape.seed, device="cpu")
    to_bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    qbits, kbits = to_bits(q[0:1]), to_bits(k[0:1])
    tokens = shape.tokens
    qb = math.ceil(tokens / 128)
    fine = tokens // 4
    samples = shape.sample_pages * 32
    rows_total = shape.batch_heads * qb
    with threadpool_limits(threads):
        t0 = time.perf_counter()
        pooled = oracle.pool(kbits)
        t_pool = time.perf_counter() - t0
        sub = qbits[:, : rows_sample * 128]
        t0 = time.perf_counter()
        cent, pops, _ = oracle.cluster(sub)
        lse, mx, den = oracle.lse(cent, pooled, 1, rows_sample)
        scores = oracle.mix(lse, pops, mx, den)
        ids, logw = oracle.sip(scores, np.full(rows_sample, 0.5, np.float32), samples)
        t_plan = time.perf_counter() - t0
        t0 = time.perf_counter()
        qf = q[0:1, : rows_sample * 128].float().numpy()
        oracle.prefill(qf, k[0:1].float().numpy(), v[0:1].float().numpy(), ids, logw)
        t_prefill = time.perf_counter() - t0
    per_row = (t_plan + t_prefill) / rows_sample
    ms = (per_row * rows_total + t_pool * shape.batch_heads) * 1e3
    return {"value": ms, "unit": "ms", "cores": threads,
            "sample": f"{rows_sample} query blocks of 1 head (IBCS+SIP+prefill) + key pooling of 1 head, "
                      f"extrapolated linearly to {rows_total} blocks / {shape.batch_heads} heads",
            "sample_seconds": t_pool + t_plan + t_prefill}


def run_reference(args, shape) -> None:
    """`--impl reference`: the reference math on the host cores (the oracle port;
    the reference's only CPU path is its PyTorch-free math, which it runs on the GPU)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    values = []
    for _ in range(args.warmup):
        cpu_sample(shape, rows_sample=2, threads=cores)
    for _ in range(args.steps):
        values.append(cpu_sample(shape, rows_sample=4, threads=cores)["value"])
    value = statistics.median(values)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "ms", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": value, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic smooth-field video tokens",
        "config": {"workload": shape.name, "batch": shape.batch, "heads": shape.heads, "tokens": shape.tokens,
                   "sample_pages": shape.sample_pages},
        "cpu_baseline": {"value": value, "unit": "ms", "cores": cores, "kind": "port",
                         "sample": "4 query blocks of 1 head per step (C/numpy restatement), extrapolated"},
        "e2e": {"value": value, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- GPU arm -----------------------------------------------------------------------

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
    parser.add_argument("--bh", type=int, default=0,
                        help="run only the first BH (batch*head) rows of the configuration (profiling)")
    args = parser.parse_args()

    from ab_attention_b200.synthetic import CONFIGS, make_inputs

    shape = CONFIGS[args.config]
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
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    bh = shape.batch_heads
    if bh % world:
        raise SystemExit(f"{bh} heads do not split over {world} GPUs")
    per = bh // world
    shard = slice(rank * per, (rank + 1) * per)
    q, k, v, text = make_inputs(shape, device=device, bh_slice=shard if world > 1 else None)
    q, k, v = (x.reshape(1, per, shape.tokens, 128).contiguous() for x in (q, k, v))
    if text is not None:
        text = tuple(t.reshape(1, per, -1, 128).contiguous() for t in text)
    tokens = shape.tokens
    qb = math.ceil(tokens / 128)
    rows_global = bh * qb
    gen = torch.Generator(device=device).manual_seed(shape.seed)
    offsets_all = torch.rand(rows_global, device=device, generator=gen)
    offsets = offsets_all[rank * per * qb:(rank + 1) * per * qb].contiguous()
    out_full = torch.empty((world * per, tokens, 128), dtype=torch.bfloat16, device=device) if world > 1 else None

    def barrier():
        if world > 1:
            dist.barrier()

    stream = torch.cuda.current_stream(device)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]

    def step(i=None, qq=q, kk=k, vv=v):
        e = ev[i] if i is not None else None
        if e:
            e[0].record(stream)
        plan = abx.build_plan(qq, kk, sample_pages=shape.sample_pages, offsets=offsets)
        if e:
            e[1].record(stream)
        o = abx.apply_plan(qq, kk, vv, plan, text_kv=text)
        if e:
            e[2].record(stream)
        if world > 1:
            dist.all_gather_into_tensor(out_full, o.reshape(per, tokens, 128))
        if e:
            e[3].record(stream)
        return o

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for i in range(args.steps):
            step(i)
        stop.record(stream)
        torch.cuda.synchronize()
    barrier()
    elapsed = start.elapsed_time(stop)
    plan_ms = statistics.median(e[0].elapsed_time(e[1]) for e in ev)
    prefill_ms = statistics.median(e[1].elapsed_time(e[2]) for e in ev)
    gather_ms = statistics.median(e[2].elapsed_time(e[3]) for e in ev)
    t = torch.tensor([elapsed, plan_ms, prefill_ms, gather_ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed, plan_ms, prefill_ms, gather_ms = t.tolist()
    ms = elapsed / args.steps

    # End to end through the public API: pinned host inputs in, output back out.
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
        hout = torch.empty(q.shape, dtype=q.dtype).pin_memory()
        h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv))
        d2h = hout.numel() * hout.element_size()

        def e2e_step():
            dq, dk, dv = (x.to(device, non_blocking=True) for x in (hq, hk, hv))
            o = step(None, dq, dk, dv)
            hout.copy_(o, non_blocking=True)
            return o

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
                   "step": "build_plan (fresh plan) + apply_plan" + (" + all_gather" if world > 1 else "")},
        "eff_tflops": eq_flops / (ms * 1e-3) / 1e12,
        "sparse_tflops": sparse_flops / (ms * 1e-3) / 1e12,
        "plan_ms": plan_ms, "prefill_ms": prefill_ms, "all_gather_ms": gather_ms,
        "plan_amortised_ms": prefill_ms + plan_ms / 4 + gather_ms,
        "roofline": {"kernel": "sparse prefill", "bound": "tensor", "achieved": achieved,
                     "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops_sustained"], "traffic": None,
                     "peak_source": peaks["source"] + " sustained bf16"},
        "gpu_launches": 5 * args.steps,
        "clocks": clocks.summary(),
        **dense,
    }
    if e2e is not None:
        line["e2e"] = e2e
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_sample(shape)
        line["cpu_baseline"]["kind"] = "port"
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
