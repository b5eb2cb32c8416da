"""GPU parity of the HT-weighted sparse prefill against the float64 oracle.

The reference runs this stage through FlashInfer's Hopper-only fa3 backend,
which cannot run here, so the oracle is a float64 evaluation of the same
sampled estimator (oracle/oracle.py: prefill). Tolerance (bf16 output):
max abs err <= 2e-2 and mean abs err <= 2e-3; LSE within 1e-2 (log2 units).
"""
import math

import numpy as np
import pytest
import torch

from ab_attention_b200 import apply_plan, build_plan, dense_attention
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
    if lse is not None:
        lerr = np.abs(_np(lse).reshape(lse_ref.shape) - lse_ref)
        assert lerr.max() <= LSE_ERR, f"lse max err {lerr.max()}"


@pytest.mark.parametrize("bh,grid,pages,sigma", [
    (2, (2, 16, 32), 2, 0.1),     # 1024 tokens, full blocks
    (1, (1, 4, 257), 4, 0.3),     # 1028 tokens: partial last query block (4 queries)
    (2, (3, 16, 40), 8, 0.1),     # 1920 tokens, 256 sampled blocks
])
def test_sparse_prefill_vs_oracle(bh, grid, pages, sigma):
    q, k, v = smooth_field(bh, *grid, seed=7, sigma=sigma, device="cuda")
    q4, k4, v4 = (x.unsqueeze(0) for x in (q, k, v))
    plan = build_plan(q4, k4, sample_pages=pages, seed=3)
    o, lse = apply_plan(q4, k4, v4, plan, return_lse=True)
    rows = plan.descriptor.shape[0]
    ids = plan.descriptor.reshape(rows, -1).cpu().numpy()
    logw = plan.log_weights.reshape(rows, -1).cpu().numpy()
    o_ref, lse_ref = oracle.prefill(_np(q), _np(k), _np(v), ids, logw)
    _check(o[0], lse[0], o_ref, lse_ref)


def test_sparse_prefill_with_text_keys():
    bh, grid = 2, (2, 16, 32)
    q, k, v = smooth_field(bh, *grid, seed=8, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(5)
    tk = torch.randn(bh, 256, 128, device="cuda", generator=gen).bfloat16()
    tv = torch.randn(bh, 256, 128, device="cuda", generator=gen).bfloat16()
    q4, k4, v4 = (x.unsqueeze(0) for x in (q, k, v))
    plan = build_plan(q4, k4, sample_pages=2, seed=3)
    o, lse = apply_plan(q4, k4, v4, plan, return_lse=True, text_kv=(tk.unsqueeze(0), tv.unsqueeze(0)))
    rows = plan.descriptor.shape[0]
    o_ref, lse_ref = oracle.prefill(_np(q), _np(k), _np(v), plan.descriptor.reshape(rows, -1).cpu().numpy(),
                                    plan.log_weights.reshape(rows, -1).cpu().numpy(), _np(tk), _np(tv))
    _check(o[0], lse[0], o_ref, lse_ref)


@pytest.mark.parametrize("tokens", [512, 1028])
def test_dense_mode_vs_oracle(tokens):
    q, k, v = smooth_field(2, 1, 1, tokens, seed=4, device="cuda")
    o, lse = dense_attention(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), return_lse=True)
    o_ref, lse_ref = oracle.dense(_np(q), _np(k), _np(v))
    _check(o[0], lse[0], o_ref, lse_ref)


def test_full_budget_converges_to_dense():
    """As the sample budget approaches the population every block becomes pi=1
    and the estimator equals dense attention (weights 0)."""
    q, k, v = smooth_field(1, 1, 2, 512, seed=6, device="cuda")
    q4, k4, v4 = (x.unsqueeze(0) for x in (q, k, v))
    fine = q.shape[1] // 4
    rows = math.ceil(q.shape[1] / 128)
    ids = torch.arange(fine, dtype=torch.int32, device="cuda").repeat(rows, 1).reshape(rows, fine // 32, 32)
    logw = torch.zeros_like(ids, dtype=torch.float32)
    o = apply_plan(q4, k4, v4, (ids, logw))
    od = dense_attention(q4, k4, v4)
    assert (o.float() - od.float()).abs().max().item() <= 1e-2


def test_sparse_prefill_matches_torch_fp32_reference():
    """The HT estimator written in plain PyTorch fp32 (gather + softmax) on the GPU."""
    bh, grid = 2, (2, 16, 64)
    q, k, v = smooth_field(bh, *grid, seed=10, device="cuda")
    q4, k4, v4 = (x.unsqueeze(0) for x in (q, k, v))
    plan = build_plan(q4, k4, sample_pages=4, seed=1)
    o = apply_plan(q4, k4, v4, plan)
    tokens = q.shape[1]
    qb = math.ceil(tokens / 128)
    ids = plan.descriptor.reshape(bh, qb, -1).long()
    w = plan.log_weights.reshape(bh, qb, -1)
    tok = (4 * ids[..., None] + torch.arange(4, device="cuda")).reshape(bh, qb, -1)
    kf, vf, qf = k.float(), v.float(), q.float()
    out = torch.empty_like(qf)
    for h in range(bh):
        for r in range(qb):
            keys = kf[h, tok[h, r]]
            vals = vf[h, tok[h, r]]
            logits = qf[h, r * 128:(r + 1) * 128] @ keys.T * (128 ** -0.5) * math.log2(math.e)
            logits = logits + w[h, r].repeat_interleave(4)[None, :]
            p = torch.softmax(logits * math.log(2), dim=-1)
            out[h, r * 128:(r + 1) * 128] = p @ vals
    err = (o[0].float() - out).abs()
    assert err.max().item() <= MAX_ERR and err.mean().item() <= MEAN_ERR


def test_torch_ops_and_paged_attention_match_python_api():
    from ab_attention_b200 import ops
    from ab_attention_b200.attention import paged_attention

    bh, grid = 2, (2, 16, 32)
    q, k, v = smooth_field(bh, *grid, seed=11, device="cuda")
    q4, k4, v4 = (x.unsqueeze(0) for x in (q, k, v))
    plan = build_plan(q4, k4, sample_pages=2, seed=9)
    o, lse = apply_plan(q4, k4, v4, plan, return_lse=True)
    o2, lse2 = paged_attention(q4, k4, v4, plan.descriptor, plan.log_weights, return_lse=True)
    assert torch.equal(o, o2) and torch.equal(lse, lse2)
    rows = plan.descriptor.shape[0]
    ids = plan.descriptor.reshape(rows, -1).contiguous()
    logw = plan.log_weights.reshape(rows, -1).contiguous()
    o3, lse3 = torch.ops.ab_attention.sparse_prefill(q, k, v, ids, logw)
    assert torch.equal(o3, o[0]) and torch.equal(lse3, lse[0])
    scores = torch.ops.ab_attention.ibcs(q4, k4)
    assert torch.equal(scores, ops.ibcs(q4, k4))
    gen = torch.Generator(device="cuda").manual_seed(9)
    offsets = torch.rand(rows, device="cuda", generator=gen)
    ids2 = torch.empty_like(ids)
    logw2 = torch.empty_like(logw)
    torch.ops.ab_attention.sip(scores, offsets, ids2, logw2)
    assert torch.equal(ids2, ids) and torch.equal(logw2, logw)
    ids3, logw3 = torch.ops.ab_attention.build_plan(q4, k4, offsets, ids.shape[1])
    assert torch.equal(ids3, ids) and torch.equal(logw3, logw)


@pytest.mark.parametrize("with_text", [False, True])
def test_host_pipeline_equals_device_path(with_text):
    """ab_attention_host (chunked copy-in / compute / copy-out) gives the device
    path's result bit for bit, including a ragged last chunk, with and without
    prompt keys."""
    from ab_attention_b200 import ab_attention_host

    q, k, v = (x.reshape(1, 5, -1, 128) for x in smooth_field(5, 2, 16, 32, seed=12, device="cuda"))
    text = None
    if with_text:
        gen = torch.Generator(device="cuda").manual_seed(6)
        text = tuple(torch.randn(1, 5, 37, 128, generator=gen, device="cuda").to(torch.bfloat16) for _ in range(2))
    want = apply_plan(q, k, v, build_plan(q, k, sample_pages=2, seed=7), text_kv=text)
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    host_text = None if text is None else tuple(t.cpu() for t in text)
    got = ab_attention_host(hq, hk, hv, sample_pages=2, seed=7, heads_per_chunk=2, text_kv=host_text)
    assert got.device.type == "cpu"
    assert torch.equal(got, want.cpu())


@pytest.mark.parametrize("with_text", [False, True])
def test_sharded_host_pipeline_equals_device_path(with_text):
    """attention_sharded_host (block copy-in / plan + prefill + gather / copy-out on
    three streams), run as one rank, gives the device path's result bit for bit
    in both the gathered device output and the host output."""
    from ab_attention_b200 import shard

    heads, chunks = 4, 2
    q, k, v = (x.reshape(1, heads, -1, 128) for x in smooth_field(heads, 2, 16, 32, seed=13, device="cuda"))
    tokens = q.shape[2]
    text = None
    if with_text:
        gen = torch.Generator(device="cuda").manual_seed(5)
        text = tuple(torch.randn(1, heads, 37, 128, generator=gen, device="cuda").to(torch.bfloat16)
                     for _ in range(2))
    offsets = shard.layer_offsets(heads, tokens, seed=3, device="cuda")
    want = apply_plan(q, k, v, build_plan(q, k, sample_pages=2, offsets=offsets), text_kv=text)
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    host_out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    out = torch.empty((heads, tokens, 128), dtype=torch.bfloat16, device="cuda")
    shard.attention_sharded_host(hq, hk, hv, offsets, out, host_out, world=1, chunks=chunks, sample_pages=2,
                                 text_kv=text)
    torch.cuda.synchronize()
    assert torch.equal(out, want[0])
    assert torch.equal(host_out, want.cpu())


@pytest.mark.parametrize("sizes,streams", [([2, 1, 1], 2), ([3, 1], 1), (4, 2)])
def test_sharded_blocks_on_alternating_streams_equal_device_path(sizes, streams):
    """attention_sharded run as one rank, with tapered or even head blocks whose
    prefills alternate between streams, writes the device path's output bit for bit
    (host pipeline likewise with uneven blocks)."""
    from ab_attention_b200 import shard

    heads = 4
    q, k, v = (x.reshape(1, heads, -1, 128) for x in smooth_field(heads, 2, 16, 32, seed=14, device="cuda"))
    tokens = q.shape[2]
    offsets = shard.layer_offsets(heads, tokens, seed=4, device="cuda")
    want = apply_plan(q, k, v, build_plan(q, k, sample_pages=2, offsets=offsets))
    out = torch.zeros((heads, tokens, 128), dtype=torch.bfloat16, device="cuda")
    shard.attention_sharded(q, k, v, offsets, out, world=1, chunks=sizes, sample_pages=2, block_streams=streams)
    torch.cuda.synchronize()
    assert torch.equal(out, want[0])
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    host_out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    out.zero_()
    shard.attention_sharded_host(hq, hk, hv, offsets, out, host_out, world=1, chunks=sizes, sample_pages=2)
    torch.cuda.synchronize()
    assert torch.equal(out, want[0]) and torch.equal(host_out, want.cpu())
