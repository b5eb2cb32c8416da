"""The reference's hot-path math in PyTorch on the host CPU.

ORACLE INFRASTRUCTURE: imported only by tests/, __graft_entry__.smoke() and
bench.py's CPU legs (the `cpu_baseline` figure and the `--impl reference`
arm), never by the shipped package. It is the stand-in for "the reference math
run in PyTorch on the box's own host cores": the reference has no CPU
implementation of its own (its IBCS/SIP kernels are CUDA, csrc/ibcs.cu and
csrc/sip.cu, and its prefill is FlashInfer's Hopper-only fa3 backend).

Each stage restates one reference stage, vectorised over query blocks, with
the reference's rounding points (bf16 centroids and scaled centroid operand,
bf16 pooled keys, fp16 centroid LSEs, float scores, double SIP masses, float
log-weights) and its selection rules (farthest-first centres with ties to the
lowest index, strict-< assignment, the certainty loop, certain units first in
ascending order, systematic draws at u + k):

    cluster  <- cluster_queries_kernel  csrc/ibcs.cu:106-238
    pool     <- pool_keys_kernel        csrc/ibcs.cu:244-266
    lse      <- ibcs_lse_kernel         csrc/ibcs.cu:270-489
    mix      <- ibcs_scores_kernel      csrc/ibcs.cu:495-538
    sip      <- sip_kernel              csrc/sip.cu:33-167
    prefill  <- paged_attention + ABSipAttention, flashinfer_backend.py:30-58,164-242

Sums run in PyTorch's order, not the GPU kernels' reduction trees, and the
exponentials are exact rather than fast-math, so results agree with the
bit-exact kernels (and with oracle/abx_oracle.c) to a tolerance. The head
dimension is a parameter (the reference fixes it at 128): configuration 0 of
the benchmark runs at D = 64 in fp32 through this module.
"""
from __future__ import annotations

import math

import torch

QUERY_BLOCK = 128
CENTROIDS = 8
KV4 = 4


def kappa(dim: int) -> float:
    """dim^-1/2 * log2(e), rounded to float (csrc/ibcs.cu:601-602 for dim = 128)."""
    return float(torch.tensor(dim ** -0.5 * 1.4426950408889634, dtype=torch.float32))


def bf16_round(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def _blocks(q: torch.Tensor):
    """[BH, S, D] -> zero-padded [rows, 128, D] query blocks and the valid mask."""
    bh, seq, dim = q.shape
    qb = math.ceil(seq / QUERY_BLOCK)
    padded = torch.nn.functional.pad(q, (0, 0, 0, qb * QUERY_BLOCK - seq))
    blocks = padded.reshape(bh * qb, QUERY_BLOCK, dim)
    n = torch.full((bh, qb), QUERY_BLOCK, dtype=torch.int64)
    n[:, -1] = seq - (qb - 1) * QUERY_BLOCK
    valid = torch.arange(QUERY_BLOCK)[None, :] < n.reshape(-1, 1)
    return blocks, valid


def cluster(q: torch.Tensor):
    """Farthest-first 8-way clustering of every 128-query block.

    Returns (centroids [rows, 8, D] f32 holding bf16 values, populations
    [rows, 8] f32, assignments [rows, 128] int64 with -1 past a partial block)."""
    blocks, valid = _blocks(q.to(torch.float32))
    rows = blocks.shape[0]
    n = valid.sum(1)
    mean = (blocks * valid[..., None]).sum(1) / n[:, None]
    neg_inf = torch.tensor(-math.inf)
    dist = torch.where(valid, ((blocks - mean[:, None]) ** 2).sum(-1), neg_inf)
    center = dist.argmax(1)  # first maximal index: ties to the lowest query
    min_dist = torch.full(valid.shape, math.inf)
    assign = torch.zeros(valid.shape, dtype=torch.int64)
    index = torch.arange(rows)
    for slot in range(CENTROIDS):
        c = blocks[index, center]
        d = ((blocks - c[:, None]) ** 2).sum(-1)
        better = valid & (d < min_dist)
        min_dist = torch.where(better, d, min_dist)
        assign = torch.where(better, torch.tensor(slot), assign)
        if slot + 1 < CENTROIDS:
            center = torch.where(valid, min_dist, neg_inf).argmax(1)
    onehot = torch.nn.functional.one_hot(assign, CENTROIDS).to(torch.float32) * valid[..., None]
    counts = onehot.sum(1)
    sums = torch.einsum("rqc,rqd->rcd", onehot, blocks)
    centroids = torch.where(counts[..., None] > 0, bf16_round(sums / counts.clamp(min=1)[..., None]),
                            torch.zeros(()))
    return centroids, counts, torch.where(valid, assign, torch.tensor(-1))


def pool(k: torch.Tensor) -> torch.Tensor:
    """Two representatives per KV4 block: bf16(0.5 * (k[4j+2t] + k[4j+2t+1])). [BH, F, 2, D]."""
    bh, seq, dim = k.shape
    pairs = k.to(torch.float32).reshape(bh, seq // KV4, 2, 2, dim)
    return bf16_round(0.5 * (pairs[:, :, :, 0] + pairs[:, :, :, 1]))


def lse(centroids: torch.Tensor, pooled: torch.Tensor, qb: int):
    """Per (row, centroid, KV4 block) the fp16 pair log2-sum-exp of the two scaled
    centroid . representative scores (+1 for the pair size each representative
    stands for), and each (row, centroid)'s log2-domain max and softmax denominator.
    Returns (lse [rows, 8, F] f32 holding fp16 values, max [rows, 8], den [rows, 8])."""
    bh, fine, _, dim = pooled.shape
    scaled = bf16_round(centroids * kappa(dim)).reshape(bh, qb * CENTROIDS, dim)
    x = torch.bmm(scaled, pooled.reshape(bh, fine * 2, dim).transpose(1, 2)) + 1.0
    x = x.reshape(bh * qb, CENTROIDS, fine, 2)
    a, b = x[..., 0], x[..., 1]
    top = torch.maximum(a, b)
    pair = top + torch.log2(torch.clamp(torch.exp2(a - top) + torch.exp2(b - top), min=1e-20))
    values = pair.to(torch.float16).to(torch.float32)
    mx = values.max(-1).values
    den = torch.exp2(values - mx[..., None]).sum(-1)
    return values, mx, den


def mix(values: torch.Tensor, populations: torch.Tensor, mx: torch.Tensor, den: torch.Tensor) -> torch.Tensor:
    """Population-weighted mixture of the eight centroid distributions: [rows, F] f32."""
    prob = torch.exp2(values - mx[..., None]) / den[..., None]
    return (populations[..., None] * prob).sum(1) / populations.sum(1, keepdim=True)


def sip(scores: torch.Tensor, offsets: torch.Tensor, samples: int):
    """Iterative pi = 1 certainty, then systematic sampling at u + k.

    scores [rows, F] f32, offsets [rows] f32 in [0, 1) -> (ids [rows, samples]
    int32, log_weights [rows, samples] f32 = -log2(pi), 0 for certain units)."""
    rows, population = scores.shape
    v = torch.clamp(scores.to(torch.float32), min=1e-30).to(torch.float64)
    certain = torch.zeros((rows, population), dtype=torch.bool)
    count = torch.zeros(rows, dtype=torch.int64)
    scale = torch.zeros(rows, dtype=torch.float64)
    active = torch.ones(rows, dtype=torch.bool)
    while True:
        total = torch.where(certain, 0.0, v).sum(1)
        scale = torch.where(active, (samples - count) / total, scale)
        newly = active[:, None] & ~certain & (v * scale[:, None] >= 1.0)
        added = newly.sum(1)
        if not bool(added.any()):
            break
        certain |= newly
        count += added
        active = added > 0
    masses = torch.where(certain, 0.0, v * scale[:, None])
    cumulative = masses.cumsum(1)
    pos = torch.arange(samples)[None, :]
    first_residual = pos >= count[:, None]
    draws = offsets.to(torch.float64)[:, None] + (pos - count[:, None]).clamp(min=0)
    picked = torch.searchsorted(cumulative.contiguous(), draws.contiguous(), right=True)
    residual = ~certain
    last = population - 1 - residual.flip(1).to(torch.int8).argmax(1)  # last residual unit
    picked = torch.minimum(picked, last[:, None])
    order = torch.sort((~certain).to(torch.int8), dim=1, stable=True).indices[:, :samples]
    ids = torch.where(first_residual, picked, order)
    raw = torch.gather(scores.to(torch.float64), 1, ids).clamp(min=1e-30)
    logw = torch.where(first_residual, -torch.log2(raw * scale[:, None]), torch.zeros((), dtype=torch.float64))
    return ids.to(torch.int32), logw.to(torch.float32)


def prefill(q, k, v, ids, log_weights, text_k=None, text_v=None, rows_per_chunk: int = 16):
    """HT-weighted sparse attention in f32: for each plan row the keys 4 * id + 0..3
    of its granules with logit shift log_weights[slot] (log2 units), then the
    always-included text keys; o = softmax_2(l) V, lse = log2 sum 2^l.
    q/k/v [BH, S, D] -> (o [BH, S, D] f32, lse [BH, S] f32)."""
    bh, seq, dim = q.shape
    qb = math.ceil(seq / QUERY_BLOCK)
    scale = kappa(dim)
    blocks, _ = _blocks(q.to(torch.float32))
    k32, v32 = k.to(torch.float32), v.to(torch.float32)
    out = torch.empty((bh * qb, QUERY_BLOCK, dim))
    lse_out = torch.empty((bh * qb, QUERY_BLOCK))
    offs = torch.arange(KV4)
    for head in range(bh):
        for r0 in range(0, qb, rows_per_chunk):
            r1 = min(qb, r0 + rows_per_chunk)
            rows = slice(head * qb + r0, head * qb + r1)
            tok = (KV4 * ids[rows].to(torch.int64)[..., None] + offs).reshape(r1 - r0, -1)
            keys, vals = k32[head][tok], v32[head][tok]
            w = log_weights[rows].to(torch.float32).repeat_interleave(KV4, dim=1)
            if text_k is not None:
                t = text_k.shape[1]
                keys = torch.cat([keys, text_k[head].to(torch.float32).expand(r1 - r0, t, dim)], 1)
                vals = torch.cat([vals, text_v[head].to(torch.float32).expand(r1 - r0, t, dim)], 1)
                w = torch.cat([w, torch.zeros(r1 - r0, t)], 1)
            logits = torch.bmm(blocks[rows], keys.transpose(1, 2)) * scale + w[:, None, :]
            m = logits.max(-1, keepdim=True).values
            p = torch.exp2(logits - m)
            total = p.sum(-1, keepdim=True)
            out[rows] = torch.bmm(p, vals) / total
            lse_out[rows] = (m + torch.log2(total))[..., 0]
    o = out.reshape(bh, qb * QUERY_BLOCK, dim)[:, :seq]
    return o, lse_out.reshape(bh, qb * QUERY_BLOCK)[:, :seq]


def build_plan(q, k, samples: int, offsets):
    """IBCS then SIP: q/k [BH, S, D] -> (ids, log_weights) [rows, samples]."""
    bh, seq, _ = q.shape
    qb = math.ceil(seq / QUERY_BLOCK)
    centroids, populations, _ = cluster(q)
    values, mx, den = lse(centroids, pool(k), qb)
    return sip(mix(values, populations, mx, den), offsets, samples)


def layer(q, k, v, samples: int, offsets, text_k=None, text_v=None):
    """One AB-attention layer on the host: a fresh plan and the sparse prefill.
    Returns (o, lse, ids, log_weights)."""
    ids, logw = build_plan(q, k, samples, offsets)
    o, lse_ = prefill(q, k, v, ids, logw, text_k, text_v)
    return o, lse_, ids, logw
