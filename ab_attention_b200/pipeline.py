"""AB-attention of a layer whose Q/K/V live in host memory.

`ab_attention_host` streams the layer through the GPU in head chunks on three
CUDA streams: the copy-in of chunk c + 1, the plan and sparse prefill of chunk
c and the copy-out of chunk c - 1 overlap, so the layer costs about the larger
of the PCIe transfers and the compute instead of their sum. Plans are
bit-identical to `build_plan` on the whole layer: the per-row uniforms are
drawn once from the seed for every head (ab_attention/attention.py:56-57) and
sliced per chunk.
"""
from __future__ import annotations

import math

import torch

from .attention import apply_plan, build_plan


@torch.no_grad()
def ab_attention_host(q, k, v, *, sample_pages=64, seed=42, out=None, heads_per_chunk=4, device=None,
                      text_kv=None):
    """``ab_attention`` for host tensors: q, k, v [B, H, N, 128] bf16 in host
    memory (pinned for overlap); returns the output in host memory (``out`` if
    given: [B, H, N, 128] bf16, pinned for overlap). ``text_kv=(text_k, text_v)``
    ([B, H, T, 128] bf16, host or device; moved to the device once) adds prompt
    keys every query block includes with weight pi = 1, as ``apply_plan``'s
    ``text_kv``. Synchronizes before returning."""
    if q.device.type != "cpu" or k.device.type != "cpu" or v.device.type != "cpu":
        raise ValueError("ab_attention_host takes host tensors")
    if q.ndim != 4 or q.shape != k.shape or q.shape != v.shape or q.dtype != torch.bfloat16 or q.shape[-1] != 128:
        raise ValueError("Q/K/V must be matching [B,H,N,128] bf16 tensors")
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    batch, heads, tokens, dim = q.shape
    bh = batch * heads
    qb = math.ceil(tokens / 128)
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    elif out.shape != q.shape or out.dtype != q.dtype or out.device.type != "cpu":
        raise ValueError("out must be a host tensor shaped like q")
    flat = [x.reshape(bh, tokens, dim) for x in (q, k, v)]
    out_flat = out.view(bh, tokens, dim)
    if text_kv is not None:
        text_k, text_v = text_kv
        if text_k.shape != text_v.shape or text_k.ndim != 4 or text_k.shape[:2] != q.shape[:2] \
                or text_k.shape[-1] != dim or text_k.dtype != q.dtype or text_v.dtype != q.dtype:
            raise ValueError("text_kv must be two [B,H,T,128] bf16 tensors matching Q's batch and heads")
    chunk = max(1, min(heads_per_chunk, bh))
    starts = list(range(0, bh, chunk))

    with torch.cuda.device(device):
        main = torch.cuda.current_stream(device)
        copy_in = torch.cuda.Stream(device)
        copy_out = torch.cuda.Stream(device)
        copy_in.wait_stream(main)  # work the caller queued before this call comes first
        generator = torch.Generator(device=device).manual_seed(seed)
        offsets = torch.rand(bh * qb, device=device, generator=generator)
        text = None
        if text_kv is not None:
            text = tuple(t.reshape(bh, -1, dim).to(device) for t in text_kv)
        # two device slots per input so chunk c + 1 lands while chunk c computes
        slots = [[torch.empty((chunk, tokens, dim), dtype=q.dtype, device=device) for _ in range(3)]
                 for _ in range(2)]
        landed = [torch.cuda.Event() for _ in range(2)]
        freed = [torch.cuda.Event() for _ in range(2)]

        def load(c):
            s = c % 2
            a, b = starts[c], min(starts[c] + chunk, bh)
            with torch.cuda.stream(copy_in):
                if c >= 2:
                    copy_in.wait_event(freed[s])  # the slot's previous chunk has been consumed
                for dst, src in zip(slots[s], flat):
                    dst[:b - a].copy_(src[a:b], non_blocking=True)
                landed[s].record(copy_in)

        load(0)
        for c in range(len(starts)):
            if c + 1 < len(starts):
                load(c + 1)
            s = c % 2
            a, b = starts[c], min(starts[c] + chunk, bh)
            n = b - a
            main.wait_event(landed[s])
            qs, ks, vs = (x[:n].unsqueeze(0) for x in slots[s])
            plan = build_plan(qs, ks, sample_pages=sample_pages, offsets=offsets[a * qb:b * qb])
            block_text = None if text is None else tuple(t[a:b].unsqueeze(0) for t in text)
            o = apply_plan(qs, ks, vs, plan, text_kv=block_text)
            freed[s].record(main)
            done = torch.cuda.Event()
            done.record(main)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(done)
                out_flat[a:b].copy_(o[0], non_blocking=True)
                o.record_stream(copy_out)
        main.wait_stream(copy_out)
        main.synchronize()
    return out
