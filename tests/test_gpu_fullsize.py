"""GPU parity of the sparse prefill at the benchmark shapes, against the float64 oracle.

The timed configurations (C1 Wan2.1-1.3B, C2 Wan2.1-14B, C3 HunyuanVideo with
256 prompt keys, C4 cube order at 16 and 256 pages) are too large for the
float64 oracle to evaluate every row in test time, so each case checks a
sample of rows of whole production-size heads: the first query block, a middle
pair (the two softmax groups of one paired CTA), the last full block, the
partial last block (80 queries at the Wan shapes, 16 at the HunyuanVideo
shape, a lone block without a pair partner in both) and rows spread over the
head. On each sampled row the output and the base-2 LSE of both the paired and
the unpaired kernel are compared with oracle.prefill_row. The plans are the
production plans of those heads: the layer's uniforms are drawn for every row
and sliced (as the multi-GPU path does), so a head's plan is the one the bench
times. Tolerances as for every prefill test: max abs err <= 2e-2 and mean abs
err <= 2e-3 on the bf16 output, LSE within 1e-2 (log2
units).
"""
import math

import numpy as np
import pytest
import torch

from ab_attention_b200 import build_plan, ops, shard
from ab_attention_b200.synthetic import CONFIGS, make_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu

MAX_ERR = 2e-2
MEAN_ERR = 2e-3
LSE_ERR = 1e-2


def _sample_rows(qb: int, extra: int, seed: int) -> list[int]:
    middle = 2 * (qb // 4)
    fixed = {0, 1, middle, middle + 1, qb - 2, qb - 1}
    rng = np.random.default_rng(seed)
    spread = [int(r) for r in rng.choice(np.arange(2, qb - 2), size=extra, replace=False)]
    return sorted(fixed | set(spread))


@pytest.mark.parametrize("config,heads,pages,extra", [
    ("wan1.3b", [0, 11], None, 4),       # C1: 591 blocks per head, the last one 80 queries
    ("wan14b", [0, 41, 79], None, 3),    # C2: first, middle and last flattened head of the layer
    ("hunyuan13b", [5, 23], None, 4),    # C3: 929 blocks (last 16 queries) + 256 prompt keys
    ("wan14b-cube", [3], 16, 6),         # C4 cube order, 16 pages (512 granules per row)
    ("wan14b-cube", [7], 256, 2),        # C4 cube order, 256 pages (8,192 granules per row)
])
def test_prefill_matches_oracle_on_sampled_rows_at_full_size(config, heads, pages, extra):
    shape = CONFIGS[config]
    pages = pages or shape.sample_pages
    tokens = shape.tokens
    qb = math.ceil(tokens / 128)
    q, k, v, text = make_inputs(shape, "cuda", bh_slice=heads)
    offsets = shard.shard_offsets(shard.layer_offsets(shape.batch_heads, tokens, shape.seed, "cuda"), tokens, heads)
    plan = build_plan(q, k, sample_pages=pages, offsets=offsets)
    rows = plan.descriptor.shape[0]
    ids = plan.descriptor.reshape(rows, -1).contiguous()
    logw = plan.log_weights.reshape(rows, -1).contiguous()
    q3, k3, v3 = (x.reshape(len(heads), tokens, 128) for x in (q, k, v))
    tk = tv = None
    if text is not None:
        tk, tv = (t.reshape(len(heads), -1, 128) for t in text)
    results = {}
    for paired in (True, False):
        o, lse = ops.sparse_prefill(q3, k3, v3, ids, logw, text_k=tk, text_v=tv, return_lse=True, paired=paired)
        torch.cuda.synchronize()
        results[paired] = (o.float().cpu().numpy(), lse.cpu().numpy())
    ids_np, logw_np = ids.cpu().numpy(), logw.cpu().numpy()
    sample = _sample_rows(qb, extra, seed=len(heads) * 1000 + pages)
    errs = {True: [], False: []}
    lerrs = {True: 0.0, False: 0.0}
    for i in range(len(heads)):
        qh, kh, vh = (x[i].double().cpu().numpy() for x in (q3, k3, v3))
        th = None if tk is None else (tk[i].double().cpu().numpy(), tv[i].double().cpu().numpy())
        for r in sample:
            row = i * qb + r
            o_ref, lse_ref = oracle.prefill_row(qh, kh, vh, ids_np[row], logw_np[row], r,
                                                *(th if th is not None else (None, None)))
            n = len(lse_ref)
            assert n == min(128, tokens - 128 * r)
            for paired in (True, False):
                o, lse = results[paired]
                errs[paired].append(np.abs(o[i, 128 * r:128 * r + n] - o_ref).ravel())
                lerrs[paired] = max(lerrs[paired], float(np.abs(lse[i, 128 * r:128 * r + n] - lse_ref).max()))
    for paired in (True, False):
        err = np.concatenate(errs[paired])
        what = "paired" if paired else "unpaired"
        assert err.max() <= MAX_ERR, f"{what}: max abs err {err.max()}"
        assert err.mean() <= MEAN_ERR, f"{what}: mean abs err {err.mean()}"
        assert lerrs[paired] <= LSE_ERR, f"{what}: lse max err {lerrs[paired]}"
