"""Head sharding across the GPUs of one node.

Every AB-attention row (head, 128-query block) depends only on its own head's
Q/K/V and its own uniform offset, so heads split across ranks with no
communication during compute. The per-row offsets are drawn once for the whole
layer from the seed (as the reference draws them before chunking,
ab_attention/attention.py:56-57) and sliced, so the plan is bit-identical for
any number of GPUs. The output is reassembled with NCCL all-gathers.

Heads are dealt to ranks in chunks so that the all-gathers overlap compute: the
layer's heads form `chunks` consecutive blocks of world * ch heads; rank r owns
heads [(c * world + r) * ch, (c * world + r + 1) * ch) of block c. A rank builds
the plan for all its heads at once, then runs the sparse prefill block by block
and all-gathers block c (straight into its place in the [BH, S, 128] output)
while block c + 1 computes.
"""
from __future__ import annotations

import math

import torch


def chunk_count(batch_heads: int, world: int, max_chunks: int = 8) -> int:
    """Largest number of head blocks <= max_chunks that divides the heads evenly.

    More blocks shorten the exposed all-gather of the last block; 8 keeps each
    block's prefill launch at several waves of CTAs at the Wan shapes."""
    if batch_heads % world:
        raise ValueError(f"{batch_heads} heads do not split evenly over {world} ranks")
    for chunks in range(max_chunks, 0, -1):
        if batch_heads % (world * chunks) == 0:
            return chunks
    return 1


def rank_heads(batch_heads: int, world: int, rank: int, chunks: int = 1) -> list[int]:
    """The flattened heads rank `rank` owns, in its local (block-major) order."""
    if batch_heads % (world * chunks):
        raise ValueError(f"{batch_heads} heads do not split into {chunks} blocks over {world} ranks")
    ch = batch_heads // (world * chunks)
    return [(c * world + rank) * ch + i for c in range(chunks) for i in range(ch)]


def head_slice(batch_heads: int, world: int, rank: int) -> slice:
    """Contiguous heads of `rank` (the one-block layout)."""
    heads = rank_heads(batch_heads, world, rank, 1)
    return slice(heads[0], heads[-1] + 1)


def layer_offsets(batch_heads: int, tokens: int, seed: int, device) -> torch.Tensor:
    """The whole layer's per-row uniforms (rows = BH * ceil(tokens/128))."""
    rows = batch_heads * math.ceil(tokens / 128)
    generator = torch.Generator(device=device).manual_seed(seed)
    return torch.rand(rows, device=device, generator=generator)


def shard_offsets(offsets: torch.Tensor, tokens: int, heads) -> torch.Tensor:
    """Rows of `heads` (a slice or a list of heads) in that order."""
    qb = math.ceil(tokens / 128)
    if isinstance(heads, slice):
        return offsets[heads.start * qb:heads.stop * qb].contiguous()
    return torch.cat([offsets[h * qb:(h + 1) * qb] for h in heads]).contiguous()


def gather_heads(local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather [BH/G, ...] shards into [BH, ...] (rank order = head order)."""
    import torch.distributed as dist

    if world == 1:
        return local
    out = torch.empty((world * local.shape[0], *local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out


def gather_block(out: torch.Tensor, local_block: torch.Tensor, world: int, block: int, group=None,
                 async_op: bool = False):
    """All-gather block `block` (each rank's [ch, ...] heads) into its place in
    `out` [BH, ...]: heads [block * world * ch, (block + 1) * world * ch)."""
    import torch.distributed as dist

    ch = local_block.shape[0]
    dst = out[block * world * ch:(block + 1) * world * ch]
    if world == 1:
        dst.copy_(local_block)
        return None
    return dist.all_gather_into_tensor(dst, local_block.contiguous(), group=group, async_op=async_op)


def attention_sharded(q, k, v, offsets, out, *, world: int, chunks: int, sample_pages: int = 64,
                      text_kv=None, group=None, timing: dict | None = None):
    """This rank's part of a head-sharded AB-attention layer.

    q, k, v: [1, per, S, 128] bf16, the rank's heads in `rank_heads(BH, world,
    rank, chunks)` order; offsets: their rows of `layer_offsets` (see
    `shard_offsets`); out: [BH, S, 128] bf16, receives every rank's output.
    The plan covers all the rank's heads in one call; the prefill runs block
    by block and block c is all-gathered on NCCL's stream while block c + 1
    computes. Returns when `out` is complete on the current stream.

    `timing` (a dict, optional) receives CUDA events recorded on the current
    stream: "plan" (start, end), "blocks" [(start, end)] around each block's
    prefill, and "tail" (after the last prefill, after the last all-gather
    has landed), whose span is the all-gather time left exposed.
    """
    from .attention import SamplePlan, apply_plan, build_plan

    per, tokens = q.shape[1], q.shape[2]
    if per % chunks:
        raise ValueError(f"{per} local heads do not split into {chunks} blocks")
    ch = per // chunks
    qb = math.ceil(tokens / 128)

    def event():
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    if timing is not None:
        timing["blocks"] = []
        plan_start = event()
    plan = build_plan(q, k, sample_pages=sample_pages, offsets=offsets)
    if timing is not None:
        timing["plan"] = (plan_start, event())
    works = []
    for c in range(chunks):
        heads = slice(c * ch, (c + 1) * ch)
        rows = slice(c * ch * qb, (c + 1) * ch * qb)
        block_plan = SamplePlan(plan.descriptor[rows], plan.log_weights[rows])
        block_text = None if text_kv is None else tuple(t[:, heads] for t in text_kv)
        start = event() if timing is not None else None
        o = apply_plan(q[:, heads], k[:, heads], v[:, heads], block_plan, text_kv=block_text)
        if timing is not None:
            timing["blocks"].append((start, event()))
        works.append(gather_block(out, o.reshape(ch, tokens, q.shape[3]), world, c, group=group, async_op=True))
    tail_start = event() if timing is not None else None
    for work in works:
        if work is not None:
            work.wait()
    if timing is not None:
        timing["tail"] = (tail_start, event())
    return out


def attention_sharded_host(q, k, v, offsets, out, host_out, *, world: int, chunks: int, sample_pages: int = 64,
                           text_kv=None, group=None):
    """`attention_sharded` for Q/K/V in host memory, with the copies overlapped.

    q, k, v: pinned host [1, per, S, 128] bf16, the rank's heads in
    `rank_heads(BH, world, rank, chunks)` order; offsets: their rows of
    `layer_offsets` on the device; out: [BH, S, 128] bf16 on the device,
    receives every rank's output; host_out: pinned host [1, per, S, 128],
    receives this rank's heads. text_kv (optional): the rank's prompt keys and
    values on the device, [1, per, T, 128] each.

    Head block c + 1 is copied in on a side stream while block c is planned,
    attended and all-gathered, and block c's own heads are copied out on a
    third stream, so the layer costs about its host transfers rather than their
    sum with the compute. The plan of each block is built from its rows of the
    layer's offsets, so it is bit-identical to `attention_sharded`'s. Every
    rank issues the same all-gathers in the same order. Returns when `out` and
    host_out are complete on the current stream.
    """
    from .attention import apply_plan, build_plan

    per, tokens, dim = q.shape[1], q.shape[2], q.shape[3]
    if per % chunks:
        raise ValueError(f"{per} local heads do not split into {chunks} blocks")
    if q.device.type != "cpu" or k.device.type != "cpu" or v.device.type != "cpu" or host_out.device.type != "cpu":
        raise ValueError("q, k, v and host_out must be host tensors")
    if host_out.shape != q.shape or host_out.dtype != q.dtype:
        raise ValueError("host_out must be shaped like q")
    ch = per // chunks
    qb = math.ceil(tokens / 128)
    device = out.device
    main = torch.cuda.current_stream(device)
    copy_in = torch.cuda.Stream(device)
    copy_out = torch.cuda.Stream(device)
    copy_in.wait_stream(main)  # work the caller queued before this call comes first
    # two device slots per input so block c + 1 lands while block c computes
    slots = [[torch.empty((1, ch, tokens, dim), dtype=q.dtype, device=device) for _ in range(3)] for _ in range(2)]
    landed = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]

    def load(c):
        s = c % 2
        with torch.cuda.stream(copy_in):
            if c >= 2:
                copy_in.wait_event(freed[s])  # the slot's previous block has been consumed
            for dst, src in zip(slots[s], (q, k, v)):
                dst.copy_(src[:, c * ch:(c + 1) * ch], non_blocking=True)
            landed[s].record(copy_in)

    works = []
    load(0)
    for c in range(chunks):
        if c + 1 < chunks:
            load(c + 1)
        s = c % 2
        main.wait_event(landed[s])
        qs, ks, vs = slots[s]
        plan = build_plan(qs, ks, sample_pages=sample_pages, offsets=offsets[c * ch * qb:(c + 1) * ch * qb])
        block_text = None if text_kv is None else tuple(t[:, c * ch:(c + 1) * ch] for t in text_kv)
        o = apply_plan(qs, ks, vs, plan, text_kv=block_text)
        freed[s].record(main)
        works.append(gather_block(out, o.reshape(ch, tokens, dim), world, c, group=group, async_op=True))
        done = torch.cuda.Event()
        done.record(main)
        with torch.cuda.stream(copy_out):
            copy_out.wait_event(done)
            host_out[:, c * ch:(c + 1) * ch].copy_(o, non_blocking=True)
            o.record_stream(copy_out)
    for work in works:
        if work is not None:
            work.wait()
    main.wait_stream(copy_out)
    return out
