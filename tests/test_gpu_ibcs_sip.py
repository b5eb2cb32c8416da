"""GPU parity of IBCS and SIP: bit-exact against the reference kernels.

Two oracles: the committed golden vectors (produced by the reference kernels
themselves, tests/golden/make_golden.py) and, at larger shapes, the reference
kernels compiled for sm_100a in oracle/_ref, run live on the same inputs.
"""
import math

import numpy as np
import pytest
import torch

from ab_attention_b200 import ops
from ab_attention_b200.attention import build_plan
from tests.helpers import CASES, bf16_bits, case_dims, f16_bits, golden, inputs, sip_edge_scores, to_device_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    from oracle.build_ref import load

    return load()


@pytest.mark.parametrize("case", list(CASES))
def test_stages_bit_exact_vs_golden(case):
    bh, tokens, qb, fine, samples = case_dims(case)
    g = golden(case)
    qbits, kbits, _ = inputs(case)
    q, k = to_device_bf16(qbits), to_device_bf16(kbits)
    cent, scaled, pops, assign = ops.cluster(q)
    np.testing.assert_array_equal(bf16_bits(cent), g["centroids"])
    np.testing.assert_array_equal(pops.cpu().numpy(), g["populations"])
    a = assign.cpu().numpy()
    counts = np.stack([(a == s).sum(axis=1) for s in range(8)], axis=1)
    np.testing.assert_array_equal(counts, g["populations"].astype(np.int64))
    pooled = ops.pool(k)
    lse, mx, den = ops.lse(scaled, pooled, qb)
    np.testing.assert_array_equal(f16_bits(lse), g["lse"])
    np.testing.assert_array_equal(mx.cpu().numpy(), g["lse_max"])
    np.testing.assert_array_equal(den.cpu().numpy(), g["lse_den"])
    scores = ops.mix(lse, pops, mx, den)
    np.testing.assert_array_equal(scores.cpu().numpy(), g["scores"])
    scores2 = ops.ibcs(q.unsqueeze(0), k.unsqueeze(0))
    np.testing.assert_array_equal(scores2.cpu().numpy(), g["scores"])
    offsets = torch.from_numpy(g["offsets"]).cuda()
    ids = torch.empty((bh * qb, samples), dtype=torch.int32, device="cuda")
    logw = torch.empty_like(ids, dtype=torch.float32)
    ops.sip(scores, offsets, ids, logw)
    np.testing.assert_array_equal(ids.cpu().numpy(), g["ids"])
    np.testing.assert_array_equal(logw.cpu().numpy(), g["log_weights"])
    plan = build_plan(q.unsqueeze(0), k.unsqueeze(0), sample_pages=samples // 32, offsets=offsets) \
        if samples % 32 == 0 else None
    if plan is not None:
        np.testing.assert_array_equal(plan.descriptor.reshape(bh * qb, -1).cpu().numpy(), g["ids"])
        np.testing.assert_array_equal(plan.log_weights.reshape(bh * qb, -1).cpu().numpy(), g["log_weights"])


@pytest.mark.parametrize("samples", [8, 64, 200])
def test_sip_edge_rows_vs_golden(samples):
    s, offsets = sip_edge_scores()
    g = golden(f"sip_edge_m{samples}")
    ids = torch.empty((s.shape[0], samples), dtype=torch.int32, device="cuda")
    logw = torch.empty((s.shape[0], samples), dtype=torch.float32, device="cuda")
    ops.sip(torch.from_numpy(s).cuda(), torch.from_numpy(offsets).cuda(), ids, logw)
    np.testing.assert_array_equal(ids.cpu().numpy(), g["ids"])
    np.testing.assert_array_equal(logw.cpu().numpy(), g["log_weights"])


def _smooth(bh, grid, seed, sigma=0.1):
    from ab_attention_b200.synthetic import smooth_field

    q, k, v = smooth_field(bh, *grid, seed=seed, sigma=sigma, device="cuda")
    return q, k, v


@pytest.mark.parametrize("bh,grid,seed,sigma", [
    (2, (21, 45, 80), 1, 0.1),   # Wan shape: F = 18,900, last q-block 80 queries
    (1, (33, 45, 80), 3, 0.1),   # Hunyuan video shape: F = 29,700, last q-block 16 queries
    (3, (5, 16, 20), 5, 0.3),
])
def test_live_reference_bit_exact(ref, bh, grid, seed, sigma):
    q, k, _ = _smooth(bh, grid, seed, sigma)
    tokens = q.shape[1]
    qb = math.ceil(tokens / 128)
    r_cent, r_pops = ref.cluster(q)
    cent, scaled, pops, _ = ops.cluster(q)
    assert torch.equal(cent.view(torch.int16), r_cent.view(bh * qb, 8, 128).view(torch.int16))
    assert torch.equal(pops, r_pops.float().view(bh * qb, 8))
    r_pool = ref.pool(k)
    pooled = ops.pool(k)
    assert torch.equal(pooled.view(torch.int16), r_pool.view(torch.int16))
    r_lse, r_mx, r_den = ref.lse(r_cent, r_pool)
    lse, mx, den = ops.lse(scaled, pooled, qb)
    assert torch.equal(lse.view(torch.int16), r_lse.view(torch.int16))
    assert torch.equal(mx, r_mx) and torch.equal(den, r_den)
    r_scores = ref.scores(r_lse, r_pops, r_mx, r_den)
    scores = ops.mix(lse, pops, mx, den)
    assert torch.equal(scores, r_scores)
    samples = 2048 if tokens > 8192 else 64
    rows = bh * qb
    gen = torch.Generator(device="cuda").manual_seed(seed)
    offsets = torch.rand(rows, device="cuda", generator=gen)
    r_ids = torch.empty((rows, samples), dtype=torch.int32, device="cuda")
    r_logw = torch.empty((rows, samples), dtype=torch.float32, device="cuda")
    ref.sip(r_scores, offsets, r_ids, r_logw)
    plan = build_plan(q.unsqueeze(0), k.unsqueeze(0), sample_pages=samples // 32, offsets=offsets)
    assert torch.equal(plan.descriptor.reshape(rows, -1), r_ids)
    assert torch.equal(plan.log_weights.reshape(rows, -1), r_logw)


def test_build_plan_seeded_offsets_match_reference(ref):
    """build_plan(seed) draws the same Philox uniforms as the reference (attention.py:56-57)."""
    q, k, _ = _smooth(2, (4, 16, 32), 9)
    tokens = q.shape[1]
    rows = 2 * math.ceil(tokens / 128)
    plan = build_plan(q.unsqueeze(0), k.unsqueeze(0), sample_pages=2, seed=1234)
    gen = torch.Generator(device="cuda").manual_seed(1234)
    offsets = torch.rand(rows, device="cuda", generator=gen)
    scores = ref.ibcs(q.unsqueeze(0), k.unsqueeze(0))
    ids = torch.empty((rows, 64), dtype=torch.int32, device="cuda")
    logw = torch.empty((rows, 64), dtype=torch.float32, device="cuda")
    ref.sip(scores, offsets, ids, logw)
    assert torch.equal(plan.descriptor.reshape(rows, -1), ids)
    assert torch.equal(plan.log_weights.reshape(rows, -1), logw)


def test_plan_properties_at_full_size():
    """Size-independent SIP properties at the Wan-1.3B shape: ids unique per row,
    certain units first and ascending with weight 0, sum of 2^-w over a row's
    draws consistent with the HT design (each weight >= 0)."""
    q, k, _ = _smooth(2, (21, 45, 80), 21)
    plan = build_plan(q.unsqueeze(0), k.unsqueeze(0), sample_pages=64, seed=42)
    ids = plan.descriptor.reshape(plan.descriptor.shape[0], -1)
    logw = plan.log_weights.reshape_as(ids)
    srt, _ = ids.sort(dim=1)
    assert bool((srt[:, 1:] != srt[:, :-1]).all()), "an id was drawn twice in one row"
    assert int(ids.min()) >= 0 and int(ids.max()) < q.shape[1] // 4
    assert bool((logw >= 0).all())
    certain = logw == 0
    # certain units form a prefix of each row
    first_residual = (~certain).int().argmax(dim=1)
    pos = torch.arange(ids.shape[1], device=ids.device)[None, :]
    assert bool((certain == (pos < first_residual[:, None])).all())


@pytest.mark.parametrize("bh,grid,pages", [(2, (3, 16, 43), 4), (1, (1, 7, 148), 8)])
def test_build_plan_equals_scores_then_sip(bh, grid, pages):
    """build_plan's SIP evaluates the mixture from the LSE rows itself; its plan is
    bit-identical to scoring first (ops.ibcs) and sampling those scores (ops.sip)."""
    from ab_attention_b200.synthetic import smooth_field
    q, k, _ = smooth_field(bh, *grid, seed=21, sigma=0.2, device="cuda")
    q4, k4 = q.unsqueeze(0), k.unsqueeze(0)
    tokens = q.shape[1]
    qb = -(-tokens // 128)
    gen = torch.Generator(device="cuda").manual_seed(8)
    offsets = torch.rand(bh * qb, device="cuda", generator=gen)
    plan = build_plan(q4, k4, sample_pages=pages, offsets=offsets)
    scores = ops.ibcs(q4, k4)
    ids = torch.empty((bh * qb, pages * 32), dtype=torch.int32, device="cuda")
    logw = torch.empty_like(ids, dtype=torch.float32)
    ops.sip(scores, offsets, ids, logw)
    np.testing.assert_array_equal(plan.descriptor.reshape(bh * qb, -1).cpu().numpy(), ids.cpu().numpy())
    np.testing.assert_array_equal(plan.log_weights.reshape(bh * qb, -1).cpu().numpy(), logw.cpu().numpy())


@pytest.mark.parametrize("bh,grid,seed,sigma", [
    (2, (21, 45, 80), 2, 0.1),   # Wan shape: 591 blocks per head, the last one 80 queries
    (1, (33, 45, 80), 3, 0.1),   # Hunyuan video shape: 929 blocks, the last one 16 queries
    (3, (5, 16, 20), 5, 0.3),    # 1,600 tokens: 13 blocks, the last one 64 queries
])
def test_cluster_assignments_bit_exact_vs_reference(ref, bh, grid, seed, sigma):
    """Every query's centroid slot equals the reference kernel's, read out of its
    shared memory (csrc/ibcs.cu:116,165-197) by the test-only hook in
    oracle/ref_ibcs_harness.cu; queries past a partial last block are -1 here."""
    q, _, _ = _smooth(bh, grid, seed, sigma)
    tokens = q.shape[1]
    qb = math.ceil(tokens / 128)
    r_cent, r_pops, r_assign = ref.cluster_assignments(q)
    cent, _, pops, assign = ops.cluster(q)
    # the hooked build still produces the reference's centroids and populations
    assert torch.equal(cent.view(torch.int16), r_cent.view(bh * qb, 8, 128).view(torch.int16))
    assert torch.equal(pops, r_pops.float().view(bh * qb, 8))
    r_assign = r_assign.view(bh * qb, 128)
    valid = torch.ones((bh * qb, 128), dtype=torch.bool, device="cuda")
    last = tokens - 128 * (qb - 1)
    valid.view(bh, qb, 128)[:, qb - 1, last:] = False
    assert torch.equal(assign[valid], r_assign[valid])
    assert bool((assign[~valid] == -1).all())
    assert int(r_assign[valid].min()) >= 0 and int(r_assign[valid].max()) < 8
