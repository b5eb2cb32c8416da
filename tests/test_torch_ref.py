"""The PyTorch restatement of the reference math (oracle/torch_ref.py), on CPU.

It is the bench's CPU baseline and reference arm and the only path for
configuration 0 (D = 64, fp32), so it is pinned here: against the golden
vectors produced by the reference kernels, against the C restatement, and
against the float64 prefill oracle; then configuration 0 runs end to end and
the sampling design's known answers are checked on it.
"""
import math

import numpy as np
import pytest
import torch

from ab_attention_b200.synthetic import CPU_PLUMBING, smooth_field
from oracle import oracle, torch_ref
from tests.helpers import CASES, bf16_bits_to_f32, case_dims, golden, inputs


def _f32(bits):
    return torch.from_numpy(bf16_bits_to_f32(bits))


@pytest.mark.parametrize("case", list(CASES))
def test_stages_match_golden(case):
    bh, tokens, qb, fine, samples = case_dims(case)
    g = golden(case)
    qbits, kbits, _ = inputs(case)
    cent, pops, assign = torch_ref.cluster(_f32(qbits))
    np.testing.assert_array_equal(pops.numpy(), g["populations"])
    want = bf16_bits_to_f32(g["centroids"])
    diff = cent.numpy() != want
    assert diff.mean() < 1e-2  # only at bf16 rounding ties of the quotient
    np.testing.assert_allclose(cent.numpy(), want, rtol=2 ** -7, atol=0)
    counts = np.stack([(assign.numpy() == s).sum(1) for s in range(8)], 1)
    np.testing.assert_array_equal(counts, g["populations"].astype(np.int64))
    values, mx, den = torch_ref.lse(torch.from_numpy(want), torch_ref.pool(_f32(kbits)), qb)
    theirs = g["lse"].view(np.float16).astype(np.float32)
    assert np.abs(values.numpy() - theirs).max() <= 2 * np.abs(theirs).max() * 2 ** -10
    np.testing.assert_allclose(mx.numpy(), g["lse_max"], rtol=0, atol=0.05)
    np.testing.assert_allclose(den.numpy(), g["lse_den"], rtol=2e-3)
    scores = torch_ref.mix(torch.from_numpy(theirs), torch.from_numpy(g["populations"]),
                           torch.from_numpy(g["lse_max"]), torch.from_numpy(g["lse_den"]))
    np.testing.assert_allclose(scores.numpy(), g["scores"], rtol=1e-5, atol=1e-12)
    ids, logw = torch_ref.sip(torch.from_numpy(g["scores"]), torch.from_numpy(g["offsets"]), samples)
    np.testing.assert_array_equal(ids.numpy(), g["ids"])
    np.testing.assert_allclose(logw.numpy(), g["log_weights"], rtol=1e-6, atol=1e-6)


def test_plan_matches_c_restatement():
    """Whole plan (IBCS + SIP) from the same inputs: the PyTorch and C restatements
    pick the same granules except where fast-math-free roundoff tips a draw."""
    case = "g2048"
    bh, tokens, qb, fine, samples = case_dims(case)
    g = golden(case)
    qbits, kbits, _ = inputs(case)
    c_ids, c_logw = oracle.sip(oracle.ibcs(qbits, kbits), g["offsets"], samples)
    ids, logw = torch_ref.build_plan(_f32(qbits), _f32(kbits), samples, torch.from_numpy(g["offsets"]))
    same = ids.numpy() == c_ids
    assert same.mean() > 0.99
    np.testing.assert_allclose(logw.numpy()[same], c_logw[same], rtol=1e-3, atol=1e-4)


def test_prefill_matches_float64_oracle():
    case = "g1028"
    bh, tokens, qb, fine, samples = case_dims(case)
    g = golden(case)
    qbits, kbits, vbits = inputs(case)
    q, k, v = (bf16_bits_to_f32(b) for b in (qbits, kbits, vbits))
    o, lse = torch_ref.prefill(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v),
                               torch.from_numpy(g["ids"]), torch.from_numpy(g["log_weights"]))
    o_ref, lse_ref = oracle.prefill(q, k, v, g["ids"], g["log_weights"])
    np.testing.assert_allclose(o.numpy(), o_ref, rtol=0, atol=1e-5)
    np.testing.assert_allclose(lse.numpy(), lse_ref, rtol=0, atol=1e-5)


def test_configuration_0_cpu_plumbing():
    """B1 H2 D64 fp32, 4x32x32 tokens, 8 pages (256 of 1,024
    granules per 128-query block), uniforms from seed 0, all on the host."""
    shape = CPU_PLUMBING
    q, k, v = smooth_field(shape.batch_heads, shape.frames, shape.height, shape.width, dim=shape.dim,
                           seed=shape.seed, sigma=shape.sigma, device="cpu", dtype=torch.float32)
    tokens, fine, samples = shape.tokens, shape.tokens // 4, shape.sample_pages * 32
    rows = shape.batch_heads * math.ceil(tokens / 128)
    offsets = torch.rand(rows, generator=torch.Generator().manual_seed(shape.seed))
    o, lse, ids, logw = torch_ref.layer(q, k, v, samples, offsets)
    assert o.shape == (2, 4096, 64) and lse.shape == (2, 4096)
    assert bool(torch.isfinite(o).all()) and bool(torch.isfinite(lse).all())
    # every row: distinct granules in range, certain units first in ascending order with weight 0
    srt = ids.sort(1).values
    assert bool((srt[:, 1:] != srt[:, :-1]).all())
    assert int(ids.min()) >= 0 and int(ids.max()) < fine
    certain = logw == 0
    first = (~certain).int().argmax(1)
    assert bool((certain == (torch.arange(samples)[None] < first[:, None])).all())
    lead = ids.long()
    for r in range(rows):
        c = int(first[r])
        assert bool((lead[r, 1:c] > lead[r, :c - 1]).all())
    assert bool((logw >= 0).all())
    # the certainty loop gives every row some pi = 1 granules (the "deterministic top pages")
    assert int(certain.sum(1).min()) > 0
    # the output is the float64 estimator over the same plan
    o_ref, lse_ref = oracle.prefill(q.numpy(), k.numpy(), v.numpy(), ids.numpy(), logw.numpy())
    np.testing.assert_allclose(o.numpy(), o_ref, rtol=0, atol=1e-4)
    np.testing.assert_allclose(lse.numpy(), lse_ref, rtol=0, atol=1e-4)
