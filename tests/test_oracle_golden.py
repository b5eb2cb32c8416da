"""The CPU oracle against the golden vectors produced by the reference kernels.

The oracle uses IEEE exp2/log2/division where the reference build uses
--use_fast_math approximations, and a float64 dot product where the reference
uses the tensor core, so some quantities agree to a tolerance instead of bit
for bit. Clustering (populations) and, given the reference's own scores, SIP
page selection are expected to agree exactly.
"""
import numpy as np
import pytest

from oracle import oracle
from tests.helpers import CASES, bf16_bits_to_f32, case_dims, golden, inputs, sip_edge_scores


@pytest.mark.parametrize("case", list(CASES))
def test_cluster_matches_golden(case):
    g = golden(case)
    qbits, _, _ = inputs(case)
    cent, pops, assign, quotient = oracle.cluster(qbits, with_quotient=True)
    np.testing.assert_array_equal(pops, g["populations"])
    # Centroids agree bit for bit except where the IEEE quotient sum/count is an
    # exact bf16 rounding tie: the GPU's fast-math division lands next to it and
    # the tie breaks the other way. Every difference must be such a tie.
    diff = cent != g["centroids"]
    ours = bf16_bits_to_f32(cent[diff]).astype(np.float64)
    theirs = bf16_bits_to_f32(g["centroids"][diff]).astype(np.float64)
    assert (np.abs(cent[diff].astype(np.int32) - g["centroids"][diff].astype(np.int32)) == 1).all()
    np.testing.assert_array_equal(quotient[diff].astype(np.float64), (ours + theirs) / 2)
    assert diff.mean() < 1e-2


@pytest.mark.parametrize("case", list(CASES))
def test_lse_and_scores_match_golden(case):
    bh, tokens, qb, fine, _ = case_dims(case)
    g = golden(case)
    _, kbits, _ = inputs(case)
    pooled = oracle.pool(kbits)
    lse, mx, den = oracle.lse(g["centroids"], pooled, bh, qb)
    ours = lse.view(np.float16).astype(np.float32)
    theirs = g["lse"].view(np.float16).astype(np.float32)
    assert np.abs(ours - theirs).max() <= 2 * np.abs(theirs).max() * 2 ** -10
    np.testing.assert_allclose(mx, g["lse_max"], rtol=0, atol=0.05)
    np.testing.assert_allclose(den, g["lse_den"], rtol=2e-3)
    scores = oracle.mix(g["lse"], g["populations"], g["lse_max"], g["lse_den"])
    np.testing.assert_allclose(scores, g["scores"], rtol=1e-5, atol=1e-12)
    full = oracle.ibcs(inputs(case)[0], kbits)
    np.testing.assert_allclose(full, g["scores"], rtol=5e-2, atol=1e-7)


@pytest.mark.parametrize("case", list(CASES))
def test_sip_matches_golden(case):
    g = golden(case)
    samples = g["ids"].shape[1]
    ids, logw = oracle.sip(g["scores"], g["offsets"], samples)
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_allclose(logw, g["log_weights"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("samples", [8, 64, 200])
def test_sip_edge_rows_match_golden(samples):
    s, offsets = sip_edge_scores()
    g = golden(f"sip_edge_m{samples}")
    ids, logw = oracle.sip(s, offsets, samples)
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_allclose(logw, g["log_weights"], rtol=1e-6, atol=1e-6)
