"""HunyuanVideo partitions (ab_attention/video.py:129-151) against the float64 oracle:
ragged prompt keys in the sparse prefill, dense cross attention (prompt queries over
video + prompt keys), the padding partition, and the whole layer on sparse and dense
steps. Tolerances as in test_gpu_prefill: max abs 2e-2, mean abs 2e-3 (bf16 output)."""
import numpy as np
import pytest
import torch

from ab_attention_b200 import apply_plan, build_plan, dense_cross_attention, hunyuan_attention
from ab_attention_b200.synthetic import smooth_field
from ab_attention_b200.video import VideoAttention, plan_seed
from oracle import oracle

pytestmark = pytest.mark.gpu

MAX_ERR = 2e-2
MEAN_ERR = 2e-3


def _np(t):
    return t.float().cpu().numpy()


def _check(o, o_ref):
    err = np.abs(_np(o).reshape(o_ref.shape) - o_ref)
    assert err.max() <= MAX_ERR, f"max abs err {err.max()}"
    assert err.mean() <= MEAN_ERR, f"mean abs err {err.mean()}"


def _rand(bh, n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(bh, n, 128, device="cuda", generator=g).bfloat16()


@pytest.mark.parametrize("text", [37, 6, 1])
def test_sparse_prefill_with_ragged_prompt_keys(text):
    q, k, v = smooth_field(2, 2, 16, 32, seed=8, device="cuda")
    tk, tv = _rand(2, text, 5), _rand(2, text, 6)
    q4, k4, v4 = (x.unsqueeze(0) for x in (q, k, v))
    plan = build_plan(q4, k4, sample_pages=2, seed=3)
    o = apply_plan(q4, k4, v4, plan, text_kv=(tk.unsqueeze(0), tv.unsqueeze(0)))
    rows = plan.descriptor.shape[0]
    o_ref, _ = oracle.prefill(_np(q), _np(k), _np(v), plan.descriptor.reshape(rows, -1).cpu().numpy(),
                              plan.log_weights.reshape(rows, -1).cpu().numpy(), _np(tk), _np(tv))
    _check(o[0], o_ref)


@pytest.mark.parametrize("nq,nk,text", [(300, 1024, 37), (130, 512, 0), (9, 0, 9), (200, 256, 128)])
def test_dense_cross_attention(nq, nk, text):
    q = _rand(2, nq, 1)
    k = _rand(2, nk, 2) if nk else None
    v = _rand(2, nk, 3) if nk else None
    extra = (_rand(2, text, 4), _rand(2, text, 5)) if text else None
    o, lse = dense_cross_attention(q.unsqueeze(0), None if k is None else k.unsqueeze(0),
                                   None if v is None else v.unsqueeze(0),
                                   extra_kv=None if extra is None else tuple(x.unsqueeze(0) for x in extra),
                                   return_lse=True)
    keys = [x for x in (k, extra[0] if extra else None) if x is not None]
    vals = [x for x in (v, extra[1] if extra else None) if x is not None]
    o_ref, lse_ref = oracle.dense(_np(q), np.concatenate([_np(x) for x in keys], 1),
                                  np.concatenate([_np(x) for x in vals], 1))
    _check(o[0], o_ref)
    assert np.abs(_np(lse[0]) - lse_ref).max() <= 1e-2


@pytest.mark.parametrize("step", [12, 5])
def test_hunyuan_layer_partitions(step):
    video, prompt, pad = 1024, 23, 9
    qv, kv_, vv = smooth_field(2, 2, 16, 32, seed=4, device="cuda")
    q = torch.cat([qv, _rand(2, prompt + pad, 7)], 1).unsqueeze(0)
    k = torch.cat([kv_, _rand(2, prompt + pad, 8)], 1).unsqueeze(0)
    v = torch.cat([vv, _rand(2, prompt + pad, 9)], 1).unsqueeze(0)
    sched = VideoAttention(2)
    sched.step = step
    out = hunyuan_attention(sched, 1, q, k, v, video, prompt)
    assert out.shape == q.shape
    qn, kn, vn = _np(q[0]), _np(k[0]), _np(v[0])
    pe = video + prompt
    if sched.is_sparse(1):
        plan = build_plan(q[:, :, :video].contiguous(), k[:, :, :video].contiguous(), sample_pages=2,
                          seed=plan_seed(1, 11))
        rows = plan.descriptor.shape[0]
        o_video, _ = oracle.prefill(qn[:, :video], kn[:, :video], vn[:, :video],
                                    plan.descriptor.reshape(rows, -1).cpu().numpy(),
                                    plan.log_weights.reshape(rows, -1).cpu().numpy(), kn[:, video:pe], vn[:, video:pe])
        o_text, _ = oracle.dense(qn[:, video:pe], kn[:, :pe], vn[:, :pe])
        _check(out[0, :, :video], o_video)
        _check(out[0, :, video:pe], o_text)
    else:
        o_main, _ = oracle.dense(qn[:, :pe], kn[:, :pe], vn[:, :pe])
        _check(out[0, :, :pe], o_main)
    o_pad, _ = oracle.dense(qn[:, pe:], kn[:, pe:], vn[:, pe:])
    _check(out[0, :, pe:], o_pad)
