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
                      text_kv=None, group=None):
    """This rank's part of a head-sharded AB-attention layer.

    q, k, v: [1, per, S, 128] bf16, the rank's heads in `rank_heads(BH, world,
    rank, chunks)` order; offsets: their rows of `layer_offsets` (see
    `shard_offsets`); out: [BH, S, 128] bf16, receives every rank's output.
    The plan covers all the rank's heads in one call; the prefill runs block
    by block and block c is all-gathered on NCCL's stream while block c + 1
    computes. Returns when `out` is complete on the current stream.
    """
    from .attention import SamplePlan, apply_plan, build_plan

    per, tokens = q.shape[1], q.shape[2]
    if per % chunks:
        raise ValueError(f"{per} local heads do not split into {chunks} blocks")
    ch = per // chunks
    qb = math.ceil(tokens / 128)
    plan = build_plan(q, k, sample_pages=sample_pages, offsets=offsets)
    works = []
    for c in range(chunks):
        heads = slice(c * ch, (c + 1) * ch)
        rows = slice(c * ch * qb, (c + 1) * ch * qb)
        block_plan = SamplePlan(plan.descriptor[rows], plan.log_weights[rows])
        block_text = None if text_kv is None else tuple(t[:, heads] for t in text_kv)
        o = apply_plan(q[:, heads], k[:, heads], v[:, heads], block_plan, text_kv=block_text)
        works.append(gather_block(out, o.reshape(ch, tokens, q.shape[3]), world, c, group=group, async_op=True))
    for work in works:
        if work is not None:
            work.wait()
    return out
