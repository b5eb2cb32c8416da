"""Device-side failure detection without a GPU fault: a bounded wait on an
mbarrier that nothing arrives at gives up, the host reads ABX_ERR_DEVICE_TIMEOUT,
clears it, and the same context keeps running the kernels correctly."""
import ctypes

import pytest
import torch

from ab_attention_b200 import _lib, apply_plan, build_plan
from ab_attention_b200.synthetic import smooth_field

pytestmark = pytest.mark.gpu

TIMEOUT = 5  # ABX_ERR_DEVICE_TIMEOUT


def _status(lib, clear):
    out = ctypes.c_int(-1)
    assert lib.abx_device_status(None, clear, ctypes.byref(out)) == 0
    return out.value


def test_expired_wait_is_reported_and_context_stays_usable():
    lib = _lib.load()
    torch.cuda.init()
    _status(lib, 1)
    q, k, v = (t.unsqueeze(0) for t in smooth_field(1, 2, 16, 32, seed=2, device="cuda"))
    plan = build_plan(q, k, sample_pages=2, seed=1)
    before = apply_plan(q, k, v, plan)
    assert lib.abx_selftest_wait_timeout(2_000_000, None) == 0  # ~1 ms at B200 clocks
    torch.cuda.synchronize()
    assert _status(lib, 1) == TIMEOUT
    assert _status(lib, 0) == 0
    after = apply_plan(q, k, v, plan)
    torch.cuda.synchronize()
    assert torch.equal(before, after)
    assert _status(lib, 0) == 0
