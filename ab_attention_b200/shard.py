"""Head sharding across the GPUs of one node.

Every AB-attention row (head, 128-query block) depends only on its own head's
Q/K/V and its own uniform offset, so heads split across ranks with no
communication during compute. Rank g owns the contiguous flattened heads
[g*BH/G, (g+1)*BH/G); the per-row offsets are drawn once for the whole layer
from the seed (as the reference draws them before chunking,
ab_attention/attention.py:56-57) and sliced, so the plan is bit-identical for
any number of GPUs. One all-gather reassembles the [BH, S, 128] output.
"""
from __future__ import annotations

import math

import torch


def head_slice(batch_heads: int, world: int, rank: int) -> slice:
    if batch_heads % world:
        raise ValueError(f"{batch_heads} heads do not split evenly over {world} ranks")
    per = batch_heads // world
    return slice(rank * per, (rank + 1) * per)


def layer_offsets(batch_heads: int, tokens: int, seed: int, device) -> torch.Tensor:
    """The whole layer's per-row uniforms (rows = BH * ceil(tokens/128))."""
    rows = batch_heads * math.ceil(tokens / 128)
    generator = torch.Generator(device=device).manual_seed(seed)
    return torch.rand(rows, device=device, generator=generator)


def shard_offsets(offsets: torch.Tensor, tokens: int, heads: slice) -> torch.Tensor:
    qb = math.ceil(tokens / 128)
    return offsets[heads.start * qb:heads.stop * qb].contiguous()


def gather_heads(local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather [BH/G, ...] shards into [BH, ...] (rank order = head order)."""
    import torch.distributed as dist

    if world == 1:
        return local
    out = torch.empty((world * local.shape[0], *local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out
