"""GPU parity of the paired sparse prefill (two adjacent query blocks per CTA
over the union of their samples) against the float64 oracle and against the
unpaired kernel, on plans built to hit each layout of the union stream:
identical rows (shared tiles only), disjoint rows (exclusive tiles only),
unequal exclusive counts, a lone last query block, text keys with a ragged
last granule, and plans with a repeated or out-of-range id (never merged).
Tolerance as for the unpaired prefill: max abs err <= 2e-2, mean abs err <=
2e-3, LSE within 1e-2 (log2 units).
"""
import numpy as np
import pytest
import torch

from ab_attention_b200 import _lib, build_plan, ops
from ab_attention_b200.synthetic import smooth_field
from oracle import oracle

pytestmark = pytest.mark.gpu

MAX_ERR = 2e-2
MEAN_ERR = 2e-3
LSE_ERR = 1e-2


def _np(t):
    return t.float().cpu().numpy()


def _check(o, lse, o_ref, lse_ref):
    err = np.abs(_np(o).reshape(o_ref.shape) - o_ref)
    assert err.max() <= MAX_ERR, f"max abs err {err.max()}"
    assert err.mean() <= MEAN_ERR, f"mean abs err {err.mean()}"
    lerr = np.abs(_np(lse).reshape(lse_ref.shape) - lse_ref)
    assert lerr.max() <= LSE_ERR, f"lse max err {lerr.max()}"


def _run_both(q, k, v, ids, logw, text=None):
    tk, tv = text if text is not None else (None, None)
    o1, l1 = ops.sparse_prefill(q, k, v, ids, logw, text_k=tk, text_v=tv, return_lse=True, paired=True)
    o0, l0 = ops.sparse_prefill(q, k, v, ids, logw, text_k=tk, text_v=tv, return_lse=True, paired=False)
    torch.cuda.synchronize()
    return (o1, l1), (o0, l0)


def _oracle(q, k, v, ids, logw, text=None):
    tk, tv = (None, None) if text is None else (_np(text[0]), _np(text[1]))
    return oracle.prefill(_np(q), _np(k), _np(v), ids.cpu().numpy(), logw.cpu().numpy(), tk, tv)


def _fields(bh, grid, seed):
    return smooth_field(bh, *grid, seed=seed, sigma=0.2, device="cuda")


def test_workspace_size_reports_pairable_shapes():
    import ctypes
    lib = _lib.load()
    size = ctypes.c_size_t(0)
    assert lib.abx_prefill_workspace_size(80, 75600, 2048, 0, ctypes.byref(size)) == 0 and size.value > 0
    assert lib.abx_prefill_workspace_size(2, 1024, 0, 0, ctypes.byref(size)) == 0 and size.value == 0


@pytest.mark.parametrize("bh,grid,pages", [
    (2, (2, 16, 32), 2),     # 1024 tokens: 8 blocks, 4 pairs per head
    (1, (1, 4, 257), 4),     # 1028 tokens: 9 blocks (a lone last block with 4 queries)
    (2, (3, 16, 40), 8),     # 1920 tokens: 15 blocks, 256 sampled granules
])
def test_paired_matches_oracle_and_unpaired(bh, grid, pages):
    q, k, v = _fields(bh, grid, seed=11)
    plan = build_plan(q.unsqueeze(0), k.unsqueeze(0), sample_pages=pages, seed=5)
    rows = plan.descriptor.shape[0]
    ids = plan.descriptor.reshape(rows, -1).contiguous()
    logw = plan.log_weights.reshape(rows, -1).contiguous()
    (o1, l1), (o0, l0) = _run_both(q, k, v, ids, logw)
    o_ref, lse_ref = _oracle(q, k, v, ids, logw)
    _check(o1, l1, o_ref, lse_ref)
    _check(o0, l0, o_ref, lse_ref)
    assert (o1.float() - o0.float()).abs().max().item() <= MAX_ERR


def _crafted(rows_per_head, heads, samples, fine, kind, seed=0):
    """Plans whose adjacent rows share everything, nothing, or part of their ids."""
    g = np.random.default_rng(seed)
    ids = np.empty((heads * rows_per_head, samples), np.int32)
    for r in range(ids.shape[0]):
        if kind == "identical":
            ids[r] = g.permutation(fine)[:samples] if r % 2 == 0 else ids[r - 1]
        elif kind == "disjoint":
            half = fine // 2
            base = 0 if r % 2 == 0 else half
            ids[r] = base + g.permutation(half)[:samples]
        else:  # uneven: row B keeps a prefix of A's ids, then its own
            if r % 2 == 0:
                ids[r] = g.permutation(fine)[:samples]
            else:
                keep = samples // 3
                rest = np.setdiff1d(np.arange(fine), ids[r - 1][:samples])
                ids[r] = np.concatenate([ids[r - 1][:keep], g.permutation(rest)[:samples - keep]])
    logw = g.uniform(0.0, 3.0, ids.shape).astype(np.float32)
    return torch.from_numpy(ids).cuda(), torch.from_numpy(logw).cuda()


@pytest.mark.parametrize("kind", ["identical", "disjoint", "uneven"])
def test_crafted_unions(kind):
    bh, grid = 2, (2, 16, 40)  # 1280 tokens: 10 blocks, 320 granules
    q, k, v = _fields(bh, grid, seed=12)
    ids, logw = _crafted(10, bh, 96, 320, kind, seed=3)
    (o1, l1), (o0, l0) = _run_both(q, k, v, ids, logw)
    o_ref, lse_ref = _oracle(q, k, v, ids, logw)
    _check(o1, l1, o_ref, lse_ref)
    _check(o0, l0, o_ref, lse_ref)


@pytest.mark.parametrize("text_tokens", [256, 37, 6, 1])
def test_paired_with_text(text_tokens):
    bh, grid = 2, (1, 8, 36)  # 288 tokens: 3 blocks (one pair and a lone block)
    q, k, v = _fields(bh, grid, seed=13)
    gen = torch.Generator(device="cuda").manual_seed(9)
    tk = torch.randn(bh, text_tokens, 128, device="cuda", generator=gen).bfloat16()
    tv = torch.randn(bh, text_tokens, 128, device="cuda", generator=gen).bfloat16()
    plan = build_plan(q.unsqueeze(0), k.unsqueeze(0), sample_pages=1, seed=2)
    rows = plan.descriptor.shape[0]
    ids = plan.descriptor.reshape(rows, -1).contiguous()
    logw = plan.log_weights.reshape(rows, -1).contiguous()
    (o1, l1), (o0, l0) = _run_both(q, k, v, ids, logw, text=(tk, tv))
    o_ref, lse_ref = _oracle(q, k, v, ids, logw, text=(tk, tv))
    _check(o1, l1, o_ref, lse_ref)
    _check(o0, l0, o_ref, lse_ref)


def test_repeated_id_is_not_merged():
    """A row naming a granule twice counts it twice (as the unpaired kernel and
    the reference's paged attention do); the pair falls back to exclusive tiles."""
    bh, grid = 1, (1, 8, 64)  # 512 tokens: 4 blocks, 128 granules
    q, k, v = _fields(bh, grid, seed=14)
    ids, logw = _crafted(4, bh, 48, 128, "uneven", seed=4)
    ids[1, 5] = ids[1, 6]  # repeated id in row B of the first pair
    ids[2, 0] = ids[3, 0]  # and a shared id so the second pair would merge
    (o1, l1), (o0, l0) = _run_both(q, k, v, ids, logw)
    o_ref, lse_ref = _oracle(q, k, v, ids, logw)
    _check(o1, l1, o_ref, lse_ref)
    _check(o0, l0, o_ref, lse_ref)


def test_out_of_range_id_reads_zeros_and_reports():
    bh, grid = 1, (1, 8, 64)
    q, k, v = _fields(bh, grid, seed=15)
    ids, logw = _crafted(4, bh, 48, 128, "uneven", seed=5)
    import ctypes
    lib = _lib.load()
    status = ctypes.c_int(0)
    lib.abx_device_status(None, 1, ctypes.byref(status))
    torch.cuda.synchronize()
    bad = ids.clone()
    bad[0, 3] = 10_000  # past the head's 128 granules
    o1, _ = ops.sparse_prefill(q, k, v, bad, logw, return_lse=True, paired=True)
    torch.cuda.synchronize()
    assert lib.abx_device_status(None, 1, ctypes.byref(status)) == 0
    assert status.value == 1  # ABX_ERR_INVALID_ARGUMENT
    o0, _ = ops.sparse_prefill(q, k, v, bad, logw, return_lse=True, paired=False)
    torch.cuda.synchronize()
    lib.abx_device_status(None, 1, ctypes.byref(status))
    # the bad granule reads zeros in both kernels: same outputs up to rounding
    assert (o1.float() - o0.float()).abs().max().item() <= MAX_ERR


@pytest.mark.parametrize("config,heads", [("wan14b", [0, 41]), ("hunyuan13b", [5])])
def test_paired_matches_unpaired_at_full_size(config, heads):
    """At the benchmark shapes (full-length rows, the production tile counts and
    stage rings) the paired kernel computes the same attention as one block per
    CTA, up to the order of the floating-point sums."""
    from ab_attention_b200.synthetic import CONFIGS, make_inputs
    shape = CONFIGS[config]
    q, k, v, text = make_inputs(shape, "cuda", bh_slice=heads)
    plan = build_plan(q, k, sample_pages=shape.sample_pages, seed=7)
    rows = plan.descriptor.shape[0]
    ids = plan.descriptor.reshape(rows, -1).contiguous()
    logw = plan.log_weights.reshape(rows, -1).contiguous()
    q3, k3, v3 = (x.reshape(-1, x.shape[2], 128) for x in (q, k, v))
    tkv = None if text is None else tuple(t.reshape(-1, t.shape[2], 128) for t in text)
    (o1, l1), (o0, l0) = _run_both(q3, k3, v3, ids, logw, text=tkv)
    diff = (o1.float() - o0.float()).abs()
    assert diff.max().item() <= MAX_ERR and diff.mean().item() <= MEAN_ERR / 4, (diff.max().item(), diff.mean().item())
    assert (l1 - l0).abs().max().item() <= LSE_ERR


def test_scatter_writes_every_row_into_every_output():
    """abx_sparse_prefill_scatter stores each row of its heads into every output
    buffer at the given head offset, bit-identical to the paired prefill, and
    touches no other head."""
    bh, grid = 3, (2, 16, 40)
    q, k, v = _fields(bh, grid, seed=16)
    plan = build_plan(q.unsqueeze(0), k.unsqueeze(0), sample_pages=2, seed=6)
    rows = plan.descriptor.shape[0]
    ids = plan.descriptor.reshape(rows, -1).contiguous()
    logw = plan.log_weights.reshape(rows, -1).contiguous()
    want, want_lse = ops.sparse_prefill(q, k, v, ids, logw, return_lse=True, paired=True)
    outs = [torch.full((5, q.shape[1], 128), 7.0, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    lse = ops.sparse_prefill_scatter(q, k, v, ids, logw, [o.data_ptr() for o in outs], head_base=1, out_heads=5,
                                     return_lse=True)
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o[1:4], want)
        assert bool((o[0] == 7.0).all()) and bool((o[4] == 7.0).all())
    assert torch.equal(lse, want_lse)
