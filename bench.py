"""Benchmark: one AB-attention layer (fresh plan + HT sparse prefill) at the
Wan2.1-14B 720p shape (B=2, H=40, 75,600 tokens, 64 sampled pages), heads
sharded over N B200 GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config wan14b] [--impl ours|reference]

A step is `build_plan` + `apply_plan` over the whole layer (on N > 1 each rank
does its share of the heads in blocks, each block all-gathered by NCCL while
the next computes). Rank 0 prints one JSON line; `value` is the whole-job layer
time in ms (max over ranks, CUDA events, inputs resident in HBM; the inputs are
larger than L2, so no flush is needed between steps). `e2e` repeats the
measurement through the public API with the step's inputs copied from pinned
host memory and the output copied back inside the timed region. `roofline` is
the prefill kernel timed alone (CUDA events, without its pair-plan launch)
against the measured burst bf16 peak, with the sustained peak beside it.

CPU legs: `cpu_baseline` (and the whole `--impl reference` arm) run the
reference's math restated in PyTorch (oracle/torch_ref.py) on every host core,
on whole heads of the layer, extrapolated linearly to the layer's heads; the
reference arm also times the reference's own IBCS/SIP CUDA kernels (built from
its sources into oracle/_ref) on the GPU as `ref_kernels_plan_ms`.
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
# from one ncu capture of the 4-head case (dram__bytes_read.sum + dram__bytes_write.sum
# = 278.78 + 61.46 MB; its 232 MB of Q/K/V exceed L2); a head's K/V stay L2-resident
# while its pairs run, so traffic scales with heads.
PREFILL_DRAM_BYTES_PER_HEAD = (278.78e6 + 61.46e6) / 4


def plan_bytes(bh: int, tokens: int, samples: int) -> float:
    """Algorithmic HBM bytes of build_plan: read Q and K once, write ids + weights."""
    rows = bh * math.ceil(tokens / 128)
    return 2.0 * bh * tokens * 128 * 2 + rows * samples * 8


def layer_flops(bh: int, tokens: int, keys_per_row: int) -> float:
    """4*D*BH*S*keys: QK^T and PV of the sparse prefill (D = 128)."""
    return 4.0 * 128 * bh * tokens * keys_per_row


def dense_flops(bh: int, tokens: int) -> float:
    return 4.0 * 128 * bh * tokens * tokens


# ---- CPU legs: the reference math in PyTorch on the host cores --------------------

def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def cpu_layer_sample(shape, heads: list[int], threads: int) -> dict:
    """The reference math in PyTorch (oracle/torch_ref.py: IBCS, SIP and the
    HT-weighted sparse prefill in fp32) on `heads` whole heads of the
    configuration with `threads` host threads. Every query block of a sampled
    head is planned and attended; ms per layer = mean seconds per head x B*H."""
    from ab_attention_b200.synthetic import make_inputs
    from oracle import torch_ref

    torch.set_num_threads(threads)
    tokens, bh = shape.tokens, shape.batch_heads
    qb = math.ceil(tokens / 128)
    seconds = []
    with torch.no_grad():
        for h in heads:
            q, k, v, text = make_inputs(shape, "cpu", bh_slice=[h])
            q, k, v = (x.reshape(1, tokens, 128) for x in (q, k, v))
            tk = tv = None
            if text is not None:
                tk, tv = (t.reshape(1, -1, 128) for t in text)
            offsets = torch.rand(qb, generator=torch.Generator().manual_seed(shape.seed * 1_000_003 + h))
            t0 = time.perf_counter()
            torch_ref.layer(q, k, v, shape.sample_pages * 32, offsets, tk, tv)
            seconds.append(time.perf_counter() - t0)
    per_head = statistics.mean(seconds)
    return {"value": per_head * bh * 1e3, "unit": "ms", "cores": threads, "kind": "port",
            "sample": f"{len(heads)} whole head(s) of {bh}: IBCS + SIP + sparse prefill of all {qb} query blocks "
                      f"of a head (the reference math in PyTorch fp32, oracle/torch_ref.py), {per_head:.2f} s per "
                      f"head on {threads} threads, extrapolated linearly to the layer's {bh} heads",
            "cpu_model": cpu_model(), "sample_seconds": sum(seconds)}


def reference_kernels_plan_ms(shape, reps: int = 3) -> dict:
    """The reference's own IBCS + SIP CUDA kernels (csrc/ibcs.cu, csrc/sip.cu,
    compiled from its sources for sm_100a into oracle/_ref) driven as its
    build_plan drives them (attention.py:56-75: uniforms for every row, heads
    in chunks that keep the LSE scratch within 1.5 GiB, _C.ibcs then _C.sip per
    chunk) over the whole layer on this GPU; CUDA events, median of `reps`."""
    from oracle.build_ref import load

    from ab_attention_b200.synthetic import make_inputs

    ref = load()
    device = torch.device("cuda", 0)
    q, k, _, _ = make_inputs(shape, device=device)
    bh, tokens = shape.batch_heads, shape.tokens
    q, k = (x.reshape(1, bh, tokens, 128) for x in (q, k))
    qb = math.ceil(tokens / 128)
    samples = shape.sample_pages * 32
    rows = bh * qb
    offsets = torch.rand(rows, device=device, generator=torch.Generator(device=device).manual_seed(shape.seed))
    ids = torch.empty((rows, samples), dtype=torch.int32, device=device)
    logw = torch.empty((rows, samples), dtype=torch.float32, device=device)
    per_chunk = max(1, (3 << 29) // (qb * 8 * (tokens // 4) * 2))

    def plan():
        for start in range(0, bh, per_chunk):
            stop = min(bh, start + per_chunk)
            scores = ref.ibcs(q[:, start:stop].contiguous(), k[:, start:stop].contiguous())
            ref.sip(scores, offsets[start * qb:stop * qb], ids[start * qb:stop * qb], logw[start * qb:stop * qb])

    plan()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        plan()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return {"ms": statistics.median(times), "heads_per_chunk": per_chunk}


def run_reference(args, shape) -> None:
    """`--impl reference`: the reference's math on the host cores. The reference
    has no CPU implementation of its own (its kernels are CUDA and its prefill is
    FlashInfer's Hopper-only fa3 backend), so this arm runs its math restated in
    PyTorch (oracle/torch_ref.py) on every host core: each step plans and
    attends one whole head of the layer (a different head each step) and the
    step's time is extrapolated to the layer's heads. With a GPU present, the
    line also carries the reference's own IBCS + SIP kernels timed on it over
    the whole layer (`ref_kernels_plan_ms`, same plan as build_plan's)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = host_cores()
    bh = shape.batch_heads
    for i in range(args.warmup):
        cpu_layer_sample(shape, [i % bh], cores)
    samples = [cpu_layer_sample(shape, [(args.warmup + i) % bh], cores) for i in range(args.steps)]
    value = statistics.median(s["value"] for s in samples)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "ms", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": value, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic smooth-field video tokens",
        "config": {"workload": shape.name, "batch": shape.batch, "heads": shape.heads, "tokens": shape.tokens,
                   "sample_pages": shape.sample_pages},
        "cpu_baseline": {"value": value, "unit": "ms", "cores": cores, "kind": "port",
                         "sample": f"per step one whole head of {bh} (IBCS + SIP + sparse prefill of all its query "
                                   f"blocks, the reference math in PyTorch fp32 on {cores} threads), extrapolated "
                                   f"linearly to the layer; median of {args.steps} steps",
                         "cpu_model": cpu_model()},
        "e2e": {"value": value, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if torch.cuda.is_available() and not args.no_ref_kernels:
        try:
            line["ref_kernels_plan_ms"] = reference_kernels_plan_ms(shape)
        except Exception as exc:  # noqa: BLE001  (the oracle build may be absent)
            line["ref_kernels_plan_ms"] = {"unavailable": str(exc)[:200]}
    print(json.dumps(line), flush=True)


# ---- GPU arm -----------------------------------------------------------------------

def phase_times_sharded(step, chunks, reps=3) -> dict:
    """Phases of a sharded step from events inside it (median of `reps` untimed
    steps): the plan, each head block's prefill, and the output reassembly left
    exposed after the last block's prefill. `step(timing)` runs one step."""
    import torch.distributed as dist

    samples = []
    for _ in range(reps):
        dist.barrier()
        timing = {}
        step(timing)
        torch.cuda.synchronize()
        samples.append(timing)
    med = statistics.median
    return {
        "plan_ms": med(t["plan"][0].elapsed_time(t["plan"][1]) for t in samples),
        "prefill_ms_per_block": [med(t["blocks"][c][0].elapsed_time(t["blocks"][c][1]) for t in samples)
                                 for c in range(len(samples[0]["blocks"]))],
        "exposed_gather_ms": med(t["tail"][0].elapsed_time(t["tail"][1]) for t in samples),
        "prefill_and_gather_ms": med(t["plan"][1].elapsed_time(t["tail"][1]) for t in samples),
    }


def prefill_kernel_times(q, k, v, offsets, shape, text, stream, reps: int = 5) -> dict | None:
    """The paired prefill's two launches timed apart on this rank's heads (CUDA
    events on the launch stream, median of `reps`): the pair-plan kernel and the
    prefill kernel. None when the shape cannot be paired."""
    import ab_attention_b200 as abx
    from ab_attention_b200 import ops

    per, tokens = q.shape[1], q.shape[2]
    plan = abx.build_plan(q, k, sample_pages=shape.sample_pages, offsets=offsets)
    rows = plan.descriptor.shape[0]
    ids = plan.descriptor.reshape(rows, -1).contiguous()
    logw = plan.log_weights.reshape(rows, -1).contiguous()
    q3, k3, v3 = (x.reshape(per, tokens, 128) for x in (q, k, v))
    tk = tv = None
    if text is not None:
        tk, tv = (t.reshape(per, -1, 128).contiguous() for t in text)
    text_tokens = 0 if tk is None else tk.shape[1]
    ws = ops.prefill_workspace(per, tokens, ids.shape[1], text_tokens, q.device)
    if ws is None:
        return None
    ops.pair_plan(ids, per, tokens, ws, text_tokens)
    ops.sparse_prefill_planned(q3, k3, v3, ids, logw, ws, text_k=tk, text_v=tv)
    torch.cuda.synchronize()
    plan_t, prefill_t = [], []
    for _ in range(reps):
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        e[0].record(stream)
        ops.pair_plan(ids, per, tokens, ws, text_tokens)
        e[1].record(stream)
        ops.sparse_prefill_planned(q3, k3, v3, ids, logw, ws, text_k=tk, text_v=tv)
        e[2].record(stream)
        torch.cuda.synchronize()
        plan_t.append(e[0].elapsed_time(e[1]))
        prefill_t.append(e[1].elapsed_time(e[2]))
    return {"pair_plan_ms": statistics.median(plan_t), "prefill_kernel_ms": statistics.median(prefill_t)}


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
    parser.add_argument("--shard-blocks", default="even", choices=["even", "taper"],
                        help="N > 1: head blocks of equal size, or tapered to one head per rank last")
    parser.add_argument("--block-streams", type=int, default=1,
                        help="N > 1: streams the head blocks' prefills alternate between")
    parser.add_argument("--gather", default="nccl", choices=["nccl", "copy", "peer"],
                        help="N > 1: reassemble the output with NCCL all-gathers of head blocks, with copy-engine "
                             "peer copies of each finished block (copy), or have the prefill store every row "
                             "into all ranks' copies over NVLink (peer)")
    parser.add_argument("--copy-streams", type=int, default=1,
                        help="N > 1 with --gather copy: streams the peer copies of a block are spread over "
                             "(1 .. N - 1)")
    parser.add_argument("--nccl-priority", default="normal", choices=["normal", "high"],
                        help="N > 1: priority of NCCL's stream")
    parser.add_argument("--no-ref-kernels", action="store_true",
                        help="reference arm: skip timing the reference's own IBCS/SIP kernels on the GPU")
    parser.add_argument("--sample-pages", type=int, default=0,
                        help="override the configuration's sampled pages per row (the C4 sweep: 16..256)")
    parser.add_argument("--sigma", type=float, default=0.0,
                        help="override the configuration's Q/K frequency scale (the C4 sweep: 0.05, 0.1, 0.3)")
    parser.add_argument("--bh", type=int, default=0,
                        help="run only the first BH (batch*head) rows of the configuration (profiling)")
    args = parser.parse_args()

    from ab_attention_b200.synthetic import CONFIGS, make_inputs

    shape = CONFIGS[args.config]
    if args.sample_pages:
        import dataclasses

        shape = dataclasses.replace(shape, name=f"{shape.name}[p={args.sample_pages}]", sample_pages=args.sample_pages)
    if args.sigma:
        import dataclasses

        shape = dataclasses.replace(shape, name=f"{shape.name}[sigma={args.sigma}]", sigma=args.sigma)
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
            options = None
            if args.nccl_priority == "high":
                # NCCL's kernels on a high-priority stream: the block scheduler places their
                # CTAs ahead of the prefill's pending ones
                options = dist.ProcessGroupNCCL.Options(is_high_priority_stream=True)
            dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device, pg_options=options)
            dist.barrier(device_ids=[local])
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)
    from ab_attention_b200 import shard

    bh = shape.batch_heads
    # head blocks on N > 1: even (the default) or tapered (largest first, one head per rank last)
    if world == 1 or args.gather == "peer":
        chunks = 1
    elif args.shard_blocks == "taper":
        chunks = shard.taper_sizes(bh // world)
    else:
        chunks = [bh // world // shard.chunk_count(bh, world)] * shard.chunk_count(bh, world)
    heads = shard.rank_heads(bh, world, rank, chunks)
    per = len(heads)
    q, k, v, text = make_inputs(shape, device=device, bh_slice=heads if world > 1 else None)
    q, k, v = (x.reshape(1, per, shape.tokens, 128).contiguous() for x in (q, k, v))
    if text is not None:
        text = tuple(t.reshape(1, per, -1, 128).contiguous() for t in text)
    tokens = shape.tokens
    offsets = shard.shard_offsets(shard.layer_offsets(bh, tokens, shape.seed, device), tokens, heads)
    gathered = torch.empty((bh, tokens, 128), dtype=torch.bfloat16, device=device) if world > 1 else None
    peers = (shard.PeerOutputs(gathered, copy_streams=args.copy_streams if args.gather == "copy" else 1)
             if world > 1 and args.gather in ("peer", "copy") else None)

    def sharded_step(qq, kk, vv, timing=None):
        if args.gather == "copy":
            return shard.attention_copied(qq, kk, vv, offsets, peers, rank=rank, world=world, chunks=chunks,
                                          sample_pages=shape.sample_pages, text_kv=text, timing=timing)
        if peers is not None:
            return shard.attention_scatter(qq, kk, vv, offsets, peers, rank=rank, world=world,
                                           sample_pages=shape.sample_pages, text_kv=text, timing=timing)
        return shard.attention_sharded(qq, kk, vv, offsets, gathered, world=world, chunks=chunks,
                                       sample_pages=shape.sample_pages, text_kv=text, timing=timing,
                                       block_streams=args.block_streams)

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
            sharded_step(qq, kk, vv)
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
        phases = phase_times_sharded(lambda timing: sharded_step(q, k, v, timing), chunks)
        plan_ms, prefill_ms = phases["plan_ms"], phases["prefill_and_gather_ms"]
    else:
        plan_ms = statistics.median(e[0].elapsed_time(e[1]) for e in ev)
        prefill_ms = statistics.median(e[1].elapsed_time(e[2]) for e in ev)
    # the prefill kernel alone (without its pair-plan launch) for the roofline
    kernel_times = prefill_kernel_times(q, k, v, offsets, shape, text, stream)
    pair_plan_ms = kernel_times["pair_plan_ms"] if kernel_times else 0.0
    prefill_kernel_ms = kernel_times["prefill_kernel_ms"] if kernel_times else prefill_ms
    t = torch.tensor([elapsed, plan_ms, prefill_ms, pair_plan_ms, prefill_kernel_ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed, plan_ms, prefill_ms, pair_plan_ms, prefill_kernel_ms = t.tolist()
    ms = elapsed / args.steps
    sharded = None
    if world > 1:
        # per-block prefill and the exposed all-gather tail, max over ranks
        tb = torch.tensor([phases["exposed_gather_ms"], *phases["prefill_ms_per_block"]], device=device)
        dist.all_reduce(tb, op=dist.ReduceOp.MAX)
        values = tb.tolist()
        sharded = {"output": {"nccl": "NCCL all-gather per block", "copy": "copy-engine peer copies per block",
                              "peer": "peer stores from the prefill"}[args.gather],
                   "head_blocks": chunks, "heads_per_rank": per, "exposed_gather_ms": values[0],
                   "prefill_ms_per_block": values[1:],
                   "note": "events inside attention_sharded on an untimed step, max over ranks; the exposed "
                           "gather is the wait for the last block's all-gather after its prefill"}

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
    achieved = prefill_flops_rank / (prefill_kernel_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": ms, "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic smooth-field video tokens (seeded), random per-head projections",
        "config": {"workload": shape.name, "batch": shape.batch, "heads": shape.heads, "tokens": tokens,
                   "grid": [shape.frames, shape.height, shape.width], "sample_pages": shape.sample_pages,
                   "sigma": shape.sigma, "cube_order": shape.cube,
                   "text_tokens": shape.text_tokens, "parallelism": f"heads{world}",
                   "l2": "inputs (Q/K/V 4.6 GB) larger than L2; no flush",
                   "step": "build_plan (fresh plan) + apply_plan"
                           + ("" if world == 1 else
                              " with every output row stored into all ranks' copies by the prefill (peer stores)"
                              if args.gather == "peer" else
                              f" in head blocks of {chunks} heads per rank, each copied to every rank by copy "
                              f"engines ({args.copy_streams} stream(s)) while the next computes"
                              if args.gather == "copy" else
                              f" in head blocks of {chunks} heads per rank, each all-gathered while the next "
                              f"computes")},
        "eff_tflops": eq_flops / (ms * 1e-3) / 1e12,
        "sparse_tflops": sparse_flops / (ms * 1e-3) / 1e12,
        "plan_ms": plan_ms, "prefill_ms": prefill_ms,
        "plan_amortised_ms": prefill_ms + plan_ms / 4,
        "roofline": {"kernel": "prefill_pair_kernel (timed alone, without the pair plan)", "bound": "tensor",
                     "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops"],
                     "peak_sustained": peaks["bf16_tflops_sustained"],
                     "frac_sustained": achieved / peaks["bf16_tflops_sustained"],
                     # the per-head figure was captured at the wan14b shape with 64 pages
                     "traffic": (PREFILL_DRAM_BYTES_PER_HEAD * per
                                 if shape.name.split("[")[0] == "wan14b" and shape.sample_pages == 64 else None),
                     "kernel_ms": prefill_kernel_ms, "pair_plan_ms": pair_plan_ms,
                     "peak_source": peaks["source"] + " bf16 (burst: a kernel timed alone; sustained beside it)"},
        "plan_roofline": {"kernels": "cluster (with the key pooling) + lse + sip (mixture evaluated inside sip)", "bound": "hbm",
                          "achieved": plan_bytes(per, tokens, shape.sample_pages * 32) / (plan_ms * 1e-3) / 1e9,
                          "peak": peaks["hbm_gbs"], "unit": "GB/s",
                          "frac": plan_bytes(per, tokens, shape.sample_pages * 32) / (plan_ms * 1e-3) / 1e9
                          / peaks["hbm_gbs"],
                          "note": "algorithmic bytes (Q, K in; plan out); the kernels are bound by the exact "
                                  "fast-math exp2/log2/division work and the double-precision SIP sums"},
        # cluster, pool, lse, sip + a pair plan and a prefill per head block per step
        # (NCCL's kernels not counted)
        "gpu_launches": (3 + 2 * (len(chunks) if isinstance(chunks, list) else 1)) * args.steps,
        "clocks": clocks.summary(),
        **dense,
    }
    if sharded is not None:
        line["sharded_phases"] = sharded
    if e2e is not None:
        line["e2e"] = e2e
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # four whole heads spread over the layer, every host core (about 10-30 s)
        picks = sorted({0, bh // 3, (2 * bh) // 3, bh - 1})
        line["cpu_baseline"] = cpu_layer_sample(shape, picks, host_cores())
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        if peers is not None:
            torch.cuda.synchronize()
            dist.barrier()
            peers.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
