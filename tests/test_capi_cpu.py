"""The C ABI library loads and exports every symbol include/abx.h declares;
host-side argument validation answers without touching a GPU."""
import ctypes
import re

import pytest

from ab_attention_b200 import _lib


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    names = _lib.header_symbols()
    assert len(names) >= 14
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_lib._SIGNATURES) == set(names), "ctypes signatures out of sync with abx.h"


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.abx_version() >= 1
    assert lib.abx_status_string(0) == b"ok"
    for code in range(1, 6):
        assert lib.abx_status_string(code) != b"unknown status"


@pytest.mark.parametrize("bh,seq,status", [
    (0, 1024, 1),          # no heads
    (2, 1026, 1),          # not a multiple of 4
    (2, -4, 1),
    (1, 4 * 32769, 2),     # more than 32768 KV4 blocks (csrc/ibcs.cu:567)
])
def test_workspace_size_rejects_bad_shapes(bh, seq, status):
    lib = _lib.load()
    out = ctypes.c_size_t(0)
    assert lib.abx_ibcs_workspace_size(bh, seq, ctypes.byref(out)) == status
    assert lib.abx_last_error()


def test_workspace_size_layout():
    lib = _lib.load()
    out = ctypes.c_size_t(0)
    bh, seq = 80, 75600
    assert lib.abx_ibcs_workspace_size(bh, seq, ctypes.byref(out)) == 0
    rows, fine = bh * 591, seq // 4
    ld = (fine + 7) // 8 * 8
    scratch = rows * 8 * ld * 2  # fp16 centroid LSEs (no block-score array)
    assert scratch < out.value < scratch + 2 * 1024 ** 3


def test_compute_entry_points_validate_before_launch():
    lib = _lib.load()
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    # samples must be inside the population
    assert lib.abx_sip(p, p, 4, 100, p, p, 100, None) == 1
    assert lib.abx_sip(p, p, 4, 100, p, p, 0, None) == 1
    # null / misaligned inputs
    assert lib.abx_ibcs_cluster(None, 1, 128, None, None, p, None, None) == 1
    assert lib.abx_ibcs_pool(ctypes.c_void_p(18), 1, 128, p, None) == 1
    # workspace must be present and aligned
    assert lib.abx_ibcs_scores(p, p, 1, 1024, p, None, 0, None) in (1, 3)
    assert lib.abx_build_plan(p, p, 1, 1024, p, 2048, p, p, None, 0, None) == 1  # samples >= F
    # prefill: negative text tokens, samples beyond F
    assert lib.abx_sparse_prefill(p, p, p, 1, 1024, p, p, 300, None, None, 0, p, None, None) == 1
    assert lib.abx_sparse_prefill(p, p, p, 1, 1024, p, p, 8, None, None, -4, p, None, None) == 1


def test_torch_ops_registered_without_cpu_kernel():
    import torch

    import ab_attention_b200  # noqa: F401  (registers torch.ops.ab_attention)

    q = torch.zeros(1, 1, 256, 128, dtype=torch.bfloat16)
    for call in (lambda: torch.ops.ab_attention.ibcs(q, q),
                 lambda: torch.ops.ab_attention.sparse_prefill(q[0], q[0], q[0],
                                                               torch.zeros(2, 32, dtype=torch.int32),
                                                               torch.zeros(2, 32))):
        with pytest.raises(NotImplementedError):
            call()


def test_python_api_refuses_cpu_tensors():
    import torch

    from ab_attention_b200 import apply_plan, build_plan

    q = torch.zeros(1, 1, 1024, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        build_plan(q, q, sample_pages=2)
    plan = (torch.zeros(8, 2, 32, dtype=torch.int32), torch.zeros(8, 2, 32))
    with pytest.raises(ValueError):
        apply_plan(q, q, q, plan)


def test_cross_prefill_validates_before_launch():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    # key token count must be a multiple of 4; samples within the keys; ids and weights together
    assert lib.abx_cross_prefill(p, 10, p, p, 6, 1, None, None, 1, None, None, 0, p, None, None) == 1
    assert lib.abx_cross_prefill(p, 10, p, p, 8, 1, None, None, 3, None, None, 0, p, None, None) == 1
    assert lib.abx_cross_prefill(p, 10, p, p, 8, 1, p, None, 2, None, None, 0, p, None, None) == 1
    # no keys at all; negative text count
    assert lib.abx_cross_prefill(p, 10, None, None, 0, 1, None, None, 0, None, None, 0, p, None, None) == 1
    assert lib.abx_cross_prefill(p, 10, p, p, 8, 1, None, None, 2, p, p, -1, p, None, None) == 1


def test_paired_prefill_workspace_and_validation():
    """abx_prefill_workspace_size sizes the pair lists (0 when a shape cannot be
    paired); abx_sparse_prefill_paired refuses a missing or short workspace
    before any launch."""
    lib = _lib.load()
    out = ctypes.c_size_t(0)
    bh, seq, samples = 80, 75600, 2048
    assert lib.abx_prefill_workspace_size(bh, seq, samples, 0, ctypes.byref(out)) == 0
    pairs = bh * ((591 + 1) // 2)
    per_pair = (2 * samples + 3 * 32 + 31) // 32 * 32 * 8  # entries + granule codes, 4 bytes each (32-granule tiles)
    assert pairs * per_pair <= out.value <= pairs * per_pair + pairs * 16 + 4096
    with_text = ctypes.c_size_t(0)
    assert lib.abx_prefill_workspace_size(bh, seq, samples, 256, ctypes.byref(with_text)) == 0
    assert with_text.value > out.value  # the text granules join every pair's list
    assert lib.abx_prefill_workspace_size(bh, seq, 0, 0, ctypes.byref(out)) == 0 and out.value == 0  # nothing to pair
    assert lib.abx_prefill_workspace_size(0, seq, samples, 0, ctypes.byref(out)) == 1
    assert lib.abx_prefill_workspace_size(bh, seq, -1, 0, ctypes.byref(out)) == 1
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    assert lib.abx_sparse_prefill_paired(p, p, p, 1, 1024, p, p, 8, None, None, 0, p, None, None, 0, None) == 3
    assert lib.abx_sparse_prefill_paired(p, p, p, 1, 1024, p, p, 8, None, None, 0, p, None, p, 64, None) == 3
    assert lib.abx_sparse_prefill_paired(p, p, p, 1, 1024, p, None, 8, None, None, 0, p, None, p, 1 << 30, None) == 1
    assert lib.abx_sparse_prefill_paired(ctypes.c_void_p(18), p, p, 1, 1024, p, p, 8, None, None, 0, p, None, p,
                                         1 << 30, None) == 1
    # negative counts are refused before the pairing decision, as the unpaired entry point does
    assert lib.abx_sparse_prefill_paired(p, p, p, 1, 1024, p, p, 8, p, p, -4, p, None, p, 1 << 30, None) == 1
    assert lib.abx_sparse_prefill_paired(p, p, p, 1, 1024, p, p, -8, None, None, 0, p, None, p, 1 << 30, None) == 1


def test_op_wrappers_check_buffers_before_passing_pointers():
    """The tensor wrappers hand raw pointers to the C ABI, so every buffer's dtype,
    exact shape and contiguity is checked first (a short ids or text tensor would
    otherwise be read past its end on the device)."""
    import torch

    from ab_attention_b200 import _lib, ops

    bf = torch.bfloat16
    q = torch.zeros(2, 256, 128, dtype=bf)            # BH 2, 256 tokens -> 4 rows
    ids = torch.zeros(4, 32, dtype=torch.int32)
    logw = torch.zeros(4, 32)
    bad = [
        (lambda: ops.sparse_prefill(q, q, q, ids[:3], logw[:3]), "ids must have shape"),
        (lambda: ops.sparse_prefill(q, q, q, ids, logw[:, :16]), "log_weights must have shape"),
        (lambda: ops.sparse_prefill(q.half(), q, q, ids, logw), "q must be torch.bfloat16"),
        (lambda: ops.sparse_prefill(q, q[:, :128], q, ids, logw), "k must have shape"),
        (lambda: ops.sparse_prefill(q, q, q, ids, logw, text_k=torch.zeros(2, 8, 128, dtype=bf),
                                    text_v=torch.zeros(2, 4, 128, dtype=bf)), "text_v must have shape"),
        (lambda: ops.sparse_prefill(q, q, q, ids.t(), logw.t()), "ids must have shape"),
        (lambda: ops.dense_prefill(q, q, q.transpose(1, 2).contiguous().transpose(1, 2)), "v must be contiguous"),
        (lambda: ops.cross_prefill(q, q, q, ids=ids, logw=logw, samples=16), "samples (16) must equal"),
        (lambda: ops.cross_prefill(q, None, None, samples=0, text_k=torch.zeros(1, 8, 128, dtype=bf),
                                   text_v=torch.zeros(1, 8, 128, dtype=bf)), "text_k must have shape"),
        (lambda: ops.lse(torch.zeros(7, 8, 128, dtype=bf), torch.zeros(2, 64, 2, 128, dtype=bf), 4),
         "scaled centroids must have shape"),
        (lambda: ops.mix(torch.zeros(4, 8, 64, dtype=torch.float16), torch.zeros(4, 8), torch.zeros(4, 8),
                         torch.zeros(3, 8)), "lse_den must have shape"),
        (lambda: ops.build_plan_into(q, q, torch.zeros(3), ids, logw, torch.zeros(16, dtype=torch.uint8)),
         "offsets must have shape"),
    ]
    for call, message in bad:
        with pytest.raises(RuntimeError, match=re.escape(message)):
            call()
    # well-formed host tensors get as far as the device check, and no further
    with pytest.raises(_lib.AbxError, match="CUDA"):
        ops.sparse_prefill(q, q, q, ids, logw)
    with pytest.raises(_lib.AbxError, match="CUDA"):
        ops.cross_prefill(q, None, None, samples=0, text_k=torch.zeros(2, 0, 128, dtype=bf),
                          text_v=torch.zeros(2, 0, 128, dtype=bf))


def test_torch_operators_are_cpp_with_meta_shapes():
    """torch.ops.ab_attention comes from the C++ TORCH_LIBRARY in libabx_torch.so; its
    Meta kernels give output shapes without data (for tracers)."""
    import torch

    import ab_attention_b200  # noqa: F401

    for name in ("ibcs", "sip", "build_plan", "sparse_prefill"):
        assert hasattr(torch.ops.ab_attention, name)
    q = torch.empty(2, 3, 1000, 128, dtype=torch.bfloat16, device="meta")
    scores = torch.ops.ab_attention.ibcs(q, q)
    assert scores.shape == (6 * 8, 250) and scores.dtype == torch.float32
    ids, logw = torch.ops.ab_attention.build_plan(q, q, torch.empty(48, device="meta"), 64)
    assert ids.shape == (48, 64) and ids.dtype == torch.int32 and logw.dtype == torch.float32
    q3 = q.reshape(6, 1000, 128)
    o, lse = torch.ops.ab_attention.sparse_prefill(q3, q3, q3, ids, logw)
    assert o.shape == q3.shape and lse.shape == (6, 1000)


def test_package_imports_before_the_operator_library_is_built(tmp_path, monkeypatch):
    """The build runs as `python -m ab_attention_b200.build`, which imports the package
    first: a checkout without libabx_torch.so must import (the operators are then absent)."""
    from ab_attention_b200 import _lib, ops

    monkeypatch.setattr(_lib, "PKG", tmp_path)
    assert ops._load_torch_ops() is False


def test_scatter_prefill_validates_outputs_before_launch():
    import ctypes

    lib = _lib.load()
    p = ctypes.c_void_p(16)
    one = (ctypes.c_void_p * 1)(16)
    # no output buffers; a null one; heads past the output; negative counts
    assert lib.abx_sparse_prefill_scatter(p, p, p, 2, 1024, p, p, 8, None, None, 0, one, 0, 0, 2, None, p,
                                          1 << 30, None) == 1
    assert lib.abx_sparse_prefill_scatter(p, p, p, 2, 1024, p, p, 8, None, None, 0, (ctypes.c_void_p * 1)(0), 1,
                                          0, 2, None, p, 1 << 30, None) == 1
    assert lib.abx_sparse_prefill_scatter(p, p, p, 2, 1024, p, p, 8, None, None, 0, one, 1, 3, 4, None, p,
                                          1 << 30, None) == 1
    assert lib.abx_sparse_prefill_scatter(p, p, p, 2, 1024, p, p, -8, None, None, 0, one, 1, 0, 2, None, p,
                                          1 << 30, None) == 1
    # IPC entry points refuse null arguments without touching the driver
    assert lib.abx_ipc_handle(None, None, None) == 1
    assert lib.abx_ipc_open(None, None) == 1
