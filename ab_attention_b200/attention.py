"""AB-Attention Q/K/V API on B200 (drop-in for ab_attention/attention.py).

`build_plan`, `apply_plan`, `ab_attention` and `SamplePlan` keep the
reference's signatures, defaults, layouts and ValueError conditions
(ab_attention/attention.py:11-102, flashinfer_backend.py:176-193). Additions:
`offsets=` on build_plan (inject the per-row uniforms), `text_kv=` on
apply_plan (always-included keys with pi = 1), and `dense_attention`.
"""
from __future__ import annotations

import math
from typing import NamedTuple

import torch

from . import ops

# IBCS scratch budget per launch: above it the heads are processed in chunks
# (the reference uses 1.5 GiB, attention.py:8; a B200 holds far more).
_WORKSPACE_BUDGET_BYTES = 40 * 1024 ** 3


class SamplePlan(NamedTuple):
    """SIP sample and log2(1/pi) weights, shaped [rows, pages, 32].

    ``descriptor``  - int32, sampled KV4 block ids (local to the head).
    ``log_weights`` - float32, log2 inverse-inclusion weights, same shape.
    ``rows`` is batch * heads * ceil(tokens / 128); ``pages`` is ``sample_pages``.
    """

    descriptor: torch.Tensor
    log_weights: torch.Tensor


def _draw_offsets(rows: int, device, seed: int) -> torch.Tensor:
    # One U[0,1) per row from the device Philox generator, drawn before any
    # head chunking (ab_attention/attention.py:56-57).
    generator = torch.Generator(device=device).manual_seed(seed)
    return torch.rand(rows, device=device, generator=generator)


@torch.no_grad()
def build_plan(q, k, *, sample_pages=64, seed=42, offsets=None):
    """Score and sample ``sample_pages * 128`` keys per 128-query block.

    Q and K: [batch, heads, tokens, 128] bf16 on one CUDA device; tokens divisible
    by 4 and larger than the sampled key count. Returns a ``SamplePlan``.
    ``offsets`` (float32 [rows]) replaces the seeded uniforms when given.
    """
    sample_pages = int(sample_pages)
    if q.ndim != 4 or q.shape != k.shape or q.shape[2] % 4:
        raise ValueError("Q/K must match [B,H,N,D] with N divisible by 4")
    if sample_pages <= 0:
        raise ValueError("sample_pages must be positive")
    if sample_pages * 128 >= q.shape[2]:
        raise ValueError("sampled key count must be smaller than the sequence length")
    ops._check_qk(q, k)

    batch_heads = q.shape[0] * q.shape[1]
    tokens, dim = q.shape[2:]
    q_blocks = math.ceil(tokens / 128)
    rows, samples = batch_heads * q_blocks, sample_pages * 32
    if offsets is None:
        offsets = _draw_offsets(rows, q.device, seed)
    elif offsets.shape != (rows,) or offsets.dtype != torch.float32 or offsets.device != q.device:
        raise ValueError(f"offsets must be float32 [{rows}] on the Q device")
    offsets = offsets.contiguous()
    flat_q = q.reshape(batch_heads, tokens, dim).contiguous()
    flat_k = k.reshape(batch_heads, tokens, dim).contiguous()

    per_head = ops.workspace_size(1, tokens)
    heads_per_chunk = max(1, min(batch_heads, _WORKSPACE_BUDGET_BYTES // per_head))
    sampled = torch.empty((rows, samples), dtype=torch.int32, device=q.device)
    log_weights = torch.empty((rows, samples), dtype=torch.float32, device=q.device)
    workspace = ops._workspace(heads_per_chunk, tokens, q.device)
    for start in range(0, batch_heads, heads_per_chunk):
        stop = min(batch_heads, start + heads_per_chunk)
        first, last = start * q_blocks, stop * q_blocks
        ops.build_plan_into(flat_q[start:stop], flat_k[start:stop], offsets[first:last],
                            sampled[first:last], log_weights[first:last], workspace)
    return SamplePlan(sampled.reshape(rows, sample_pages, 32), log_weights.reshape(rows, sample_pages, 32))


def _check_qkv(q, k, v):
    if q.ndim != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("Q/K/V must have the same [B,H,N,D] shape")
    if q.device != k.device or q.device != v.device:
        raise ValueError("Q/K/V must be on the same CUDA device")
    if q.device.type != "cuda":
        raise ValueError("B200 attention requires CUDA tensors")
    if q.dtype != torch.bfloat16 or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("the B200 backend requires BF16 Q/K/V")
    if q.shape[-1] != 128 or q.shape[2] % 4:
        raise ValueError("B200 attention requires head_dim=128 and N divisible by 4")


@torch.no_grad()
def paged_attention(q, k, v, descriptor, log_weights, *, return_lse=False, text_kv=None):
    """Weighted sparse attention over a plan's KV4 ids (flashinfer_backend.py:164-242).

    Same signature, checks and outputs as the reference's FlashInfer adapter;
    the work is one tcgen05 kernel launch. ``text_kv=(text_k, text_v)``
    ([B,H,T,128] bf16, any T) appends T keys that every query block always
    includes with weight pi = 1. The optional base-2 LSE is [batch, heads, tokens]
    float32.
    """
    _check_qkv(q, k, v)
    batch, heads, tokens, dim = q.shape
    batch_heads = batch * heads
    rows = batch_heads * math.ceil(tokens / 128)
    if (descriptor.ndim != 3 or descriptor.shape != log_weights.shape
            or descriptor.shape[0] != rows or descriptor.shape[-1] != 32):
        raise ValueError(f"descriptor and log_weights must share [{rows}, pages, 32] shape")
    if descriptor.device != q.device or log_weights.device != q.device:
        raise ValueError("descriptor and log_weights must be on the Q device")
    text_k = text_v = None
    if text_kv is not None:
        text_k, text_v = text_kv
        if (text_k.shape != text_v.shape or text_k.ndim != 4 or text_k.shape[:2] != q.shape[:2]
                or text_k.shape[-1] != dim or text_k.shape[2] == 0):
            raise ValueError("text_kv must be two [B,H,T,128] tensors with T > 0")
        if text_k.dtype != q.dtype or text_v.dtype != q.dtype or text_k.device != q.device:
            raise ValueError("text_kv must be BF16 on the Q device")
        text_k = text_k.reshape(batch_heads, -1, dim).contiguous()
        text_v = text_v.reshape(batch_heads, -1, dim).contiguous()
    ids = descriptor.reshape(rows, -1).to(torch.int32).contiguous()
    weights = log_weights.reshape(rows, -1).to(torch.float32).contiguous()
    out, lse = ops.sparse_prefill(q.reshape(batch_heads, tokens, dim).contiguous(),
                                  k.reshape(batch_heads, tokens, dim).contiguous(),
                                  v.reshape(batch_heads, tokens, dim).contiguous(),
                                  ids, weights, text_k=text_k, text_v=text_v, return_lse=return_lse)
    out = out.reshape_as(q)
    if not return_lse:
        return out
    return out, lse.reshape(batch, heads, tokens)


@torch.no_grad()
def apply_plan(q, k, v, plan, *, return_lse=False, text_kv=None):
    """HT-weighted sparse attention of Q over the plan's sampled KV4 blocks
    (attention.py:85-96): ``paged_attention(q, k, v, *plan)``.

    A plan can be reused across denoising steps while the shape and device stay
    the same. See ``paged_attention`` for ``text_kv`` and the LSE.
    """
    return paged_attention(q, k, v, *plan, return_lse=return_lse, text_kv=text_kv)


@torch.no_grad()
def ab_attention(q, k, v, *, sample_pages=64, seed=42):
    """AB-Attention with a fresh sampling plan; output has Q's shape and dtype."""
    return apply_plan(q, k, v, build_plan(q, k, sample_pages=sample_pages, seed=seed))


@torch.no_grad()
def dense_attention(q, k, v, *, return_lse=False):
    """Dense softmax attention (scale 128^-0.5) through the same prefill kernel."""
    _check_qkv(q, k, v)
    batch, heads, tokens, dim = q.shape
    bh = batch * heads
    out, lse = ops.dense_prefill(q.reshape(bh, tokens, dim).contiguous(), k.reshape(bh, tokens, dim).contiguous(),
                                 v.reshape(bh, tokens, dim).contiguous(), return_lse=return_lse)
    out = out.reshape_as(q)
    return (out, lse.reshape(batch, heads, tokens)) if return_lse else out


@torch.no_grad()
def dense_cross_attention(q, k, v, *, extra_kv=None, return_lse=False):
    """Softmax attention (scale 128^-0.5) of q [B,H,Nq,128] over every key of
    k/v [B,H,Nk,128] (Nk % 4 == 0; k = v = None for none) followed by every key
    of ``extra_kv=(k2, v2)`` [B,H,T,128] (any T). One launch of the prefill
    kernel; used for the HunyuanVideo text and padding partitions."""
    if q.ndim != 4 or q.dtype != torch.bfloat16 or q.shape[-1] != 128 or q.device.type != "cuda":
        raise ValueError("q must be [B,H,N,128] bf16 on a CUDA device")
    batch, heads, tokens, dim = q.shape
    bh = batch * heads
    def flat(x):
        if x.shape[:2] != q.shape[:2] or x.shape[-1] != dim or x.dtype != q.dtype or x.device != q.device:
            raise ValueError("keys must be [B,H,N,128] bf16 on the Q device")
        return x.reshape(bh, x.shape[2], dim).contiguous()
    k3 = v3 = None
    if k is not None:
        if k.shape != v.shape or k.shape[2] % 4:
            raise ValueError("k and v must match with a token count divisible by 4")
        k3, v3 = flat(k), flat(v)
    tk = tv = None
    if extra_kv is not None:
        tk, tv = (flat(x) for x in extra_kv)
        if tk.shape != tv.shape:
            raise ValueError("extra keys and values must match")
    samples = 0 if k3 is None else k3.shape[1] // 4
    out, lse = ops.cross_prefill(q.reshape(bh, tokens, dim).contiguous(), k3, v3, samples=samples,
                                 text_k=tk, text_v=tv, return_lse=return_lse)
    out = out.reshape_as(q)
    return (out, lse.reshape(batch, heads, tokens)) if return_lse else out
