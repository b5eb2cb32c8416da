"""abx_build_plan_static: the allocation-free build_plan entry point.

It exists for callers that cannot call cudaMalloc (their device memory belongs
to another allocator or is reserved up front, or cudaMalloc's implicit
synchronisation is not acceptable on their path); its scratch is a fixed
256 MiB device array inside libabx. This file is collected last, so a failure
here stops a -x run only after every other test has run.

Checked through the C ABI against abx_build_plan (caller workspace), bit for
bit, on two calls in a row with different inputs, so the second call also
shows that the contents the first call left in the shared array do not leak
into its result.
"""
import ctypes
import math

import pytest
import torch

from ab_attention_b200 import _lib, ops
from ab_attention_b200.synthetic import smooth_field


def _plan_with_workspace(lib, q, k, offsets, samples):
    bh, seq, _ = q.shape
    rows = bh * math.ceil(seq / 128)
    ids = torch.empty((rows, samples), dtype=torch.int32, device=q.device)
    logw = torch.empty((rows, samples), dtype=torch.float32, device=q.device)
    ws = torch.empty(ops.workspace_size(bh, seq), dtype=torch.uint8, device=q.device)
    _lib.check(lib.abx_build_plan(_lib.ptr(q), _lib.ptr(k), bh, seq, _lib.ptr(offsets), samples, _lib.ptr(ids),
                                  _lib.ptr(logw), _lib.ptr(ws), ws.numel(), _lib.stream_of(q)), "abx_build_plan")
    return ids, logw


def _plan_static(lib, q, k, offsets, samples):
    bh, seq, _ = q.shape
    rows = bh * math.ceil(seq / 128)
    ids = torch.empty((rows, samples), dtype=torch.int32, device=q.device)
    logw = torch.empty((rows, samples), dtype=torch.float32, device=q.device)
    _lib.check(lib.abx_build_plan_static(_lib.ptr(q), _lib.ptr(k), bh, seq, _lib.ptr(offsets), samples,
                                         _lib.ptr(ids), _lib.ptr(logw), _lib.stream_of(q)), "abx_build_plan_static")
    return ids, logw


@pytest.mark.gpu
@pytest.mark.parametrize("grid,bh,samples", [
    ((2, 16, 64), 3, 96),      # every head in one pass
    ((21, 45, 80), 2, 2048),   # Wan shape: one head per pass (about 190 MB of scratch each)
    ((4, 64, 64), 30, 512),    # 16,384 tokens, ~10.7 MB per head: 24 heads, then a ragged pass of 6
])
def test_static_scratch_matches_workspace_entry_point(grid, bh, samples):
    lib = _lib.load()
    torch.cuda.set_device(0)
    for call, seed in enumerate((31, 32)):
        q, k, _ = smooth_field(bh, *grid, seed=seed, device="cuda")
        rows = bh * math.ceil(q.shape[1] / 128)
        gen = torch.Generator(device="cuda").manual_seed(seed)
        offsets = torch.rand(rows, device="cuda", generator=gen)
        want_ids, want_logw = _plan_with_workspace(lib, q, k, offsets, samples)
        got_ids, got_logw = _plan_static(lib, q, k, offsets, samples)
        torch.cuda.synchronize()
        assert torch.equal(got_ids, want_ids), f"call {call}: ids differ"
        assert torch.equal(got_logw, want_logw), f"call {call}: log weights differ"


def test_static_scratch_rejects_inputs_beyond_its_size():
    """Runs without a GPU: the size check answers before any CUDA call."""
    lib = _lib.load()
    assert lib.abx_static_scratch_bytes() == 256 << 20
    p = ctypes.c_void_p(256)
    # one head of 118,800 tokens needs about 0.45 GB of scratch: rejected before any launch
    status = lib.abx_build_plan_static(p, p, 1, 118800, p, 2272, p, p, None)
    assert status == 3
    assert b"scratch" in lib.abx_last_error()
