"""Known-answer properties of SIP / Horvitz-Thompson and the cube layout, on the CPU oracle.

(i)   after certainty the inclusion probabilities sum to the sample count;
(ii)  over a grid of offsets u the inclusion frequency of each unit equals pi,
      and no unit is drawn twice in one row;
(iii) the HT estimate of a total is unbiased over the offset grid;
(iv)  certain units come first, ascending, with log-weight 0;
(vii) cube permutation composed with its inverse is the identity.
"""
import numpy as np
import pytest
import torch

from ab_attention_b200.layout import cube_layout
from oracle import oracle


def _pi(scores, samples):
    """Inclusion probabilities after iterative certainty (csrc/sip.cu:62-96)."""
    v = np.maximum(scores.astype(np.float64), 1e-30)
    certain = np.zeros(v.shape, bool)
    while True:
        scale = (samples - certain.sum()) / v[~certain].sum()
        new = (~certain) & (v * scale >= 1.0)
        if not new.any():
            break
        certain |= new
    return np.where(certain, 1.0, v * scale)


@pytest.fixture(scope="module")
def row():
    rng = np.random.default_rng(0)
    s = rng.gamma(0.5, size=400).astype(np.float32)
    s[[3, 50, 51]] = [40.0, 25.0, 12.0]
    return s / s.sum()


def test_inclusion_probabilities_sum_to_budget(row):
    pi = _pi(row, 40)
    assert abs(pi.sum() - 40) < 1e-9
    assert (pi <= 1 + 1e-12).all()


def test_inclusion_frequency_and_uniqueness(row):
    samples, grid = 40, 2000
    offsets = (np.arange(grid, dtype=np.float64) + 0.5) / grid
    scores = np.tile(row, (grid, 1))
    ids, logw = oracle.sip(scores, offsets.astype(np.float32), samples)
    for r in range(grid):
        assert len(np.unique(ids[r])) == samples
    freq = np.bincount(ids.reshape(-1), minlength=row.size) / grid
    pi = _pi(row, samples)
    assert np.abs(freq - pi).max() < 2.0 / grid + 1e-9
    # weights are log2(1/pi)
    np.testing.assert_allclose(2.0 ** -logw[0].astype(np.float64), pi[ids[0]], rtol=1e-5)


def test_ht_total_is_unbiased():
    # inclusion probabilities bounded away from 0, so a fine offset grid
    # approximates the expectation over u ~ U[0, 1) closely
    rng = np.random.default_rng(3)
    row = rng.uniform(0.5, 1.5, 100).astype(np.float32)
    row[[7, 60]] = [30.0, 12.0]
    samples, grid = 12, 20000
    offsets = ((np.arange(grid) + 0.5) / grid).astype(np.float32)
    y = rng.standard_normal(row.size)
    ids, logw = oracle.sip(np.tile(row, (grid, 1)), offsets, samples)
    estimates = (y[ids] * 2.0 ** logw.astype(np.float64)).sum(axis=1)
    assert abs(estimates.mean() - y.sum()) < 1e-2 * np.abs(y).sum()


def test_certain_units_first_ascending_with_zero_weight(row):
    ids, logw = oracle.sip(row[None, :], np.float32([0.3]), 40)
    pi = _pi(row, 40)
    n_certain = int((pi >= 1.0).sum())
    assert n_certain >= 3
    assert (logw[0, :n_certain] == 0).all()
    assert (np.diff(ids[0, :n_certain]) > 0).all()
    assert (logw[0, n_certain:] > 0).all()


@pytest.mark.parametrize("t,h,w", [(21, 45, 80), (33, 45, 80), (3, 5, 7), (4, 4, 4)])
def test_cube_layout_is_a_permutation(t, h, w):
    order, inverse = cube_layout(t, h, w)
    n = t * h * w
    assert order.numel() == n
    assert torch.equal(order[inverse], torch.arange(n))
    assert torch.equal(order.sort().values, torch.arange(n))
    np.testing.assert_array_equal(order.numpy(), oracle.cube_order(t, h, w))
    # first cube = the 4x4x4 corner in (t, h, w) raster order
    if t >= 4 and h >= 4 and w >= 4:
        first = order[:64].numpy()
        tt, hh, ww = np.unravel_index(first, (t, h, w))
        assert tt.max() < 4 and hh.max() < 4 and ww.max() < 4


def test_prefill_oracle_full_budget_equals_dense():
    rng = np.random.default_rng(2)
    q, k, v = (rng.standard_normal((1, 256, 128)).astype(np.float32) for _ in range(3))
    ids = np.tile(np.arange(64, dtype=np.int32), (2, 1))
    o, lse = oracle.prefill(q, k, v, ids, np.zeros_like(ids, dtype=np.float32))
    od, lsed = oracle.dense(q, k, v)
    np.testing.assert_allclose(o, od, atol=1e-10)
    np.testing.assert_allclose(lse, lsed, atol=1e-10)
