"""Tensor-level wrappers over the libabx C ABI (the custom-op layer).

These replace the reference's pybind module `ab_attention._C` (csrc/bindings.cpp:3-8)
and FlashInfer adapter (ab_attention/flashinfer_backend.py:164-242). Every op
runs on the tensors' device and the current CUDA stream, allocates its outputs
with the torch caching allocator, and raises on any nonzero status. There is
no CPU implementation.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

HEAD_DIM = 128
QUERY_BLOCK = 128
KV4 = 4
CENTROIDS = 8


def _as3(x: torch.Tensor) -> torch.Tensor:
    """[B,H,N,D] or [BH,N,D] -> contiguous [BH,N,D]."""
    if x.ndim == 4:
        x = x.reshape(x.shape[0] * x.shape[1], x.shape[2], x.shape[3])
    return x.contiguous()


def _expect(t: torch.Tensor | None, name: str, shape, dtype: torch.dtype) -> None:
    """`t` must be a contiguous tensor of exactly this shape and dtype: the C ABI
    takes raw pointers, so a short or mistyped buffer would be read past its end."""
    if t is None:
        raise RuntimeError(f"{name} is required")
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype} (got {t.dtype})")
    if tuple(t.shape) != tuple(shape):
        raise RuntimeError(f"{name} must have shape {list(shape)} (got {list(t.shape)})")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _one_device(*tensors: torch.Tensor | None) -> None:
    present = [t for t in tensors if t is not None]
    _lib.require_cuda(*present)
    if any(t.device != present[0].device for t in present):
        raise RuntimeError("all tensors must be on one CUDA device")


def _check_attention_inputs(q3, k3, v3, ids=None, logw=None, text_k=None, text_v=None, *, kv_tokens=None):
    """q3 [BH,Nq,128] bf16; k3/v3 [BH,Nk,128] bf16 (Nk = Nq unless given; both None
    when kv_tokens is 0); ids int32 and logw float32 [BH*ceil(Nq/128), samples];
    text_k/text_v [BH,T,128] bf16 with T >= 1."""
    if q3 is None or q3.ndim != 3:
        raise RuntimeError("q must be [batch*heads, tokens, 128]")
    bh, q_tokens, _ = q3.shape
    _expect(q3, "q", (bh, q_tokens, HEAD_DIM), torch.bfloat16)
    if not (kv_tokens == 0 and k3 is None and v3 is None):
        nk = q_tokens if kv_tokens is None else kv_tokens
        _expect(k3, "k", (bh, nk, HEAD_DIM), torch.bfloat16)
        _expect(v3, "v", (bh, nk, HEAD_DIM), torch.bfloat16)
    if (ids is None) != (logw is None):
        raise RuntimeError("ids and log_weights are given together")
    if ids is not None:
        rows = bh * math.ceil(q_tokens / QUERY_BLOCK)
        if ids.ndim != 2:
            raise RuntimeError("ids must be [rows, samples]")
        _expect(ids, "ids", (rows, ids.shape[1]), torch.int32)
        _expect(logw, "log_weights", (rows, ids.shape[1]), torch.float32)
    if (text_k is None) != (text_v is None):
        raise RuntimeError("text_k and text_v are given together")
    if text_k is not None:
        if text_k.ndim != 3 or text_k.shape[1] == 0:
            raise RuntimeError("text keys must be [batch*heads, T, 128] with T >= 1")
        _expect(text_k, "text_k", (bh, text_k.shape[1], HEAD_DIM), torch.bfloat16)
        _expect(text_v, "text_v", (bh, text_k.shape[1], HEAD_DIM), torch.bfloat16)
    _one_device(q3, k3, v3, ids, logw, text_k, text_v)


def _check_qk(q: torch.Tensor, k: torch.Tensor) -> None:
    _lib.require_cuda(q, k)
    if q.device != k.device:
        raise RuntimeError("q and k must use the same CUDA device")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        raise RuntimeError("IBCS requires bfloat16 q/k")
    if q.shape[-1] != HEAD_DIM:
        raise RuntimeError("IBCS requires head_dim=128")


def workspace_size(batch_heads: int, tokens: int) -> int:
    out = ctypes.c_size_t(0)
    lib = _lib.load()
    _lib.check(lib.abx_ibcs_workspace_size(batch_heads, tokens, ctypes.byref(out)), "abx_ibcs_workspace_size")
    return out.value


def _workspace(batch_heads: int, tokens: int, device) -> torch.Tensor:
    return torch.empty(workspace_size(batch_heads, tokens), dtype=torch.uint8, device=device)


# ---- IBCS stages (parity) ------------------------------------------------------

def cluster(q: torch.Tensor):
    """q [BH,S,128] bf16 -> (centroids bf16 [rows,8,128], scaled bf16 [rows,8,128],
    populations f32 [rows,8], assignments i32 [rows,128])."""
    q3 = _as3(q)
    _check_qk(q3, q3)
    bh, seq, _ = q3.shape
    rows = bh * math.ceil(seq / QUERY_BLOCK)
    cent = torch.empty((rows, CENTROIDS, HEAD_DIM), dtype=torch.bfloat16, device=q3.device)
    scaled = torch.empty_like(cent)
    pops = torch.empty((rows, CENTROIDS), dtype=torch.float32, device=q3.device)
    assign = torch.empty((rows, QUERY_BLOCK), dtype=torch.int32, device=q3.device)
    lib = _lib.load()
    with torch.cuda.device(q3.device):
        _lib.check(lib.abx_ibcs_cluster(_lib.ptr(q3), bh, seq, _lib.ptr(cent), _lib.ptr(scaled), _lib.ptr(pops),
                                        _lib.ptr(assign), _lib.stream_of(q3)), "abx_ibcs_cluster")
    return cent, scaled, pops, assign


def pool(k: torch.Tensor) -> torch.Tensor:
    """k [BH,S,128] bf16 -> pooled key representatives bf16 [BH,S/4,2,128]."""
    k3 = _as3(k)
    _check_qk(k3, k3)
    bh, seq, _ = k3.shape
    out = torch.empty((bh, seq // KV4, 2, HEAD_DIM), dtype=torch.bfloat16, device=k3.device)
    lib = _lib.load()
    with torch.cuda.device(k3.device):
        _lib.check(lib.abx_ibcs_pool(_lib.ptr(k3), bh, seq, _lib.ptr(out), _lib.stream_of(k3)), "abx_ibcs_pool")
    return out


def lse(scaled: torch.Tensor, pooled: torch.Tensor, q_blocks: int):
    """scaled centroids [BH*qb,8,128], pooled [BH,F,2,128] -> (lse fp16 [rows,8,F], max f32 [rows,8], den f32 [rows,8])."""
    if pooled.ndim != 4:
        raise RuntimeError("pooled must be [batch*heads, tokens/4, 2, 128]")
    bh, fine = pooled.shape[0], pooled.shape[1]
    rows = bh * q_blocks
    _expect(pooled, "pooled", (bh, fine, 2, HEAD_DIM), torch.bfloat16)
    _expect(scaled, "scaled centroids", (rows, CENTROIDS, HEAD_DIM), torch.bfloat16)
    _one_device(scaled, pooled)
    out = torch.empty((rows, CENTROIDS, fine), dtype=torch.float16, device=pooled.device)
    mx = torch.empty((rows, CENTROIDS), dtype=torch.float32, device=pooled.device)
    den = torch.empty_like(mx)
    lib = _lib.load()
    with torch.cuda.device(pooled.device):
        _lib.check(lib.abx_ibcs_lse(_lib.ptr(scaled), _lib.ptr(pooled), bh, q_blocks, fine,
                                    _lib.ptr(out), _lib.ptr(mx), _lib.ptr(den), _lib.stream_of(pooled)),
                   "abx_ibcs_lse")
    return out, mx, den


def mix(lse_: torch.Tensor, populations: torch.Tensor, lse_max: torch.Tensor, lse_den: torch.Tensor):
    """Population-weighted mixture -> scores f32 [rows, F]."""
    if lse_.ndim != 3:
        raise RuntimeError("lse must be [rows, 8, F]")
    rows, _, fine = lse_.shape
    _expect(lse_, "lse", (rows, CENTROIDS, fine), torch.float16)
    pops = populations.to(torch.float32).contiguous()
    _expect(pops, "populations", (rows, CENTROIDS), torch.float32)
    _expect(lse_max, "lse_max", (rows, CENTROIDS), torch.float32)
    _expect(lse_den, "lse_den", (rows, CENTROIDS), torch.float32)
    _one_device(lse_, pops, lse_max, lse_den)
    out = torch.empty((rows, fine), dtype=torch.float32, device=lse_.device)
    lib = _lib.load()
    with torch.cuda.device(lse_.device):
        _lib.check(lib.abx_ibcs_mix(_lib.ptr(lse_), _lib.ptr(pops), _lib.ptr(lse_max),
                                    _lib.ptr(lse_den), rows, fine, _lib.ptr(out),
                                    _lib.stream_of(lse_)), "abx_ibcs_mix")
    return out


# ---- reference native ops ----------------------------------------------------------

def ibcs(q: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """`_C.ibcs(q, k)` (csrc/ibcs.cu:549-617): q/k bf16 [B,H,S,128] -> scores f32 [B*H*qb, S/4]."""
    _check_qk(q, k)
    if q.shape != k.shape or q.ndim != 4:
        raise RuntimeError("q and k must have matching [batch, heads, tokens, 128] shapes")
    q3, k3 = _as3(q), _as3(k)
    bh, seq, _ = q3.shape
    rows = bh * math.ceil(seq / QUERY_BLOCK)
    scores = torch.empty((rows, seq // KV4), dtype=torch.float32, device=q.device)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        ws = _workspace(bh, seq, q.device)
        _lib.check(lib.abx_ibcs_scores(_lib.ptr(q3), _lib.ptr(k3), bh, seq, _lib.ptr(scores), _lib.ptr(ws),
                                       ws.numel(), _lib.stream_of(q3)), "abx_ibcs_scores")
    return scores


def sip(scores: torch.Tensor, offsets: torch.Tensor, ids: torch.Tensor, logs: torch.Tensor) -> None:
    """`_C.sip(scores, offsets, ids, logs)` (csrc/sip.cu:170-199): writes ids/logs in place."""
    _lib.require_cuda(scores, offsets, ids, logs)
    if not (offsets.device == scores.device == ids.device == logs.device):
        raise RuntimeError("all SIP tensors must share a CUDA device")
    if (scores.dtype != torch.float32 or offsets.dtype != torch.float32 or ids.dtype != torch.int32
            or logs.dtype != torch.float32):
        raise RuntimeError("SIP requires float32 scores/offsets/weights and int32 ids")
    if scores.ndim != 2 or offsets.ndim != 1 or ids.ndim != 2 or ids.shape != logs.shape:
        raise RuntimeError("expected scores [rows,N], offsets [rows], ids/weights [rows,samples]")
    if not (scores.is_contiguous() and offsets.is_contiguous() and ids.is_contiguous() and logs.is_contiguous()):
        raise RuntimeError("SIP tensors must be contiguous")
    if not (scores.shape[0] == offsets.shape[0] == ids.shape[0]):
        raise RuntimeError("row counts must agree")
    lib = _lib.load()
    with torch.cuda.device(scores.device):
        _lib.check(lib.abx_sip(_lib.ptr(scores), _lib.ptr(offsets), scores.shape[0], scores.shape[1], _lib.ptr(ids),
                               _lib.ptr(logs), ids.shape[1], _lib.stream_of(scores)), "abx_sip")


def build_plan_into(q3: torch.Tensor, k3: torch.Tensor, offsets: torch.Tensor, ids: torch.Tensor,
                    logw: torch.Tensor, workspace: torch.Tensor) -> None:
    """Fused IBCS + SIP for contiguous [BH,S,128] q/k into [rows, samples] ids/logw."""
    if q3.ndim != 3 or ids.ndim != 2:
        raise RuntimeError("expected q/k [batch*heads, tokens, 128] and ids/log_weights [rows, samples]")
    bh, seq, _ = q3.shape
    rows = bh * math.ceil(seq / QUERY_BLOCK)
    _expect(q3, "q", (bh, seq, HEAD_DIM), torch.bfloat16)
    _expect(k3, "k", (bh, seq, HEAD_DIM), torch.bfloat16)
    _expect(offsets, "offsets", (rows,), torch.float32)
    _expect(ids, "ids", (rows, ids.shape[1]), torch.int32)
    _expect(logw, "log_weights", (rows, ids.shape[1]), torch.float32)
    _expect(workspace, "workspace", (workspace.numel(),), torch.uint8)
    _one_device(q3, k3, offsets, ids, logw, workspace)
    lib = _lib.load()
    with torch.cuda.device(q3.device):
        _lib.check(lib.abx_build_plan(_lib.ptr(q3), _lib.ptr(k3), bh, seq, _lib.ptr(offsets), ids.shape[-1],
                                      _lib.ptr(ids), _lib.ptr(logw), _lib.ptr(workspace), workspace.numel(),
                                      _lib.stream_of(q3)), "abx_build_plan")


def sparse_prefill(q3, k3, v3, ids, logw, *, text_k=None, text_v=None, return_lse=False, paired=True):
    """HT-weighted sparse prefill over [BH,S,128] bf16 q/k/v; ids/logw [rows, samples].

    ``paired`` (default) serves two adjacent query blocks per CTA from one gather
    of the union of their samples (abx_sparse_prefill_paired); False runs one
    query block per CTA (abx_sparse_prefill). Both compute the same attention.
    """
    _check_attention_inputs(q3, k3, v3, ids, logw, text_k, text_v)
    bh, seq, _ = q3.shape
    samples = ids.shape[-1]
    o = torch.empty_like(q3)
    lse_ = torch.empty((bh, seq), dtype=torch.float32, device=q3.device) if return_lse else None
    text_tokens = 0 if text_k is None else text_k.shape[1]
    lib = _lib.load()
    with torch.cuda.device(q3.device):
        ws_bytes = ctypes.c_size_t(0)
        if paired:
            _lib.check(lib.abx_prefill_workspace_size(bh, seq, samples, text_tokens, ctypes.byref(ws_bytes)),
                       "abx_prefill_workspace_size")
        if ws_bytes.value:
            ws = torch.empty(ws_bytes.value, dtype=torch.uint8, device=q3.device)
            _lib.check(lib.abx_sparse_prefill_paired(_lib.ptr(q3), _lib.ptr(k3), _lib.ptr(v3), bh, seq,
                                                     _lib.ptr(ids), _lib.ptr(logw), samples, _lib.ptr(text_k),
                                                     _lib.ptr(text_v), text_tokens, _lib.ptr(o), _lib.ptr(lse_),
                                                     _lib.ptr(ws), ws_bytes.value, _lib.stream_of(q3)),
                       "abx_sparse_prefill_paired")
        else:
            _lib.check(lib.abx_sparse_prefill(_lib.ptr(q3), _lib.ptr(k3), _lib.ptr(v3), bh, seq, _lib.ptr(ids),
                                              _lib.ptr(logw), samples, _lib.ptr(text_k), _lib.ptr(text_v),
                                              text_tokens, _lib.ptr(o), _lib.ptr(lse_), _lib.stream_of(q3)),
                       "abx_sparse_prefill")
    return o, lse_


def prefill_workspace(bh: int, seq: int, samples: int, text_tokens: int, device) -> torch.Tensor | None:
    """Workspace for the paired prefill's union lists, or None when the shape
    cannot be paired (abx_prefill_workspace_size reports 0)."""
    size = ctypes.c_size_t(0)
    lib = _lib.load()
    _lib.check(lib.abx_prefill_workspace_size(bh, seq, samples, text_tokens, ctypes.byref(size)),
               "abx_prefill_workspace_size")
    return torch.empty(size.value, dtype=torch.uint8, device=device) if size.value else None


def pair_plan(ids: torch.Tensor, bh: int, seq: int, workspace: torch.Tensor, text_tokens: int = 0) -> None:
    """Union lists of each pair of adjacent query blocks for `ids` [rows, samples]
    into `workspace` (from prefill_workspace); a plan reused over several calls
    builds them once and then runs sparse_prefill_planned."""
    rows = bh * math.ceil(seq / QUERY_BLOCK)
    if ids.ndim != 2:
        raise RuntimeError("ids must be [rows, samples]")
    _expect(ids, "ids", (rows, ids.shape[1]), torch.int32)
    _expect(workspace, "workspace", (workspace.numel(),), torch.uint8)
    _one_device(ids, workspace)
    lib = _lib.load()
    with torch.cuda.device(ids.device):
        _lib.check(lib.abx_pair_plan(_lib.ptr(ids), bh, seq, ids.shape[1], text_tokens, _lib.ptr(workspace),
                                     workspace.numel(), _lib.stream_of(ids)), "abx_pair_plan")


def sparse_prefill_planned(q3, k3, v3, ids, logw, workspace, *, text_k=None, text_v=None, return_lse=False):
    """The paired prefill from union lists already written by pair_plan for these ids."""
    _check_attention_inputs(q3, k3, v3, ids, logw, text_k, text_v)
    _expect(workspace, "workspace", (workspace.numel(),), torch.uint8)
    bh, seq, _ = q3.shape
    o = torch.empty_like(q3)
    lse_ = torch.empty((bh, seq), dtype=torch.float32, device=q3.device) if return_lse else None
    text_tokens = 0 if text_k is None else text_k.shape[1]
    lib = _lib.load()
    with torch.cuda.device(q3.device):
        _lib.check(lib.abx_sparse_prefill_paired_planned(
            _lib.ptr(q3), _lib.ptr(k3), _lib.ptr(v3), bh, seq, _lib.ptr(ids), _lib.ptr(logw), ids.shape[1],
            _lib.ptr(text_k), _lib.ptr(text_v), text_tokens, _lib.ptr(o), _lib.ptr(lse_), _lib.ptr(workspace),
            workspace.numel(), _lib.stream_of(q3)), "abx_sparse_prefill_paired_planned")
    return o, lse_


def sparse_prefill_scatter(q3, k3, v3, ids, logw, outs, *, head_base: int, out_heads: int, text_k=None,
                           text_v=None, return_lse=False):
    """The paired prefill of [BH,S,128] q/k/v writing its rows straight into each
    buffer of `outs` (device addresses, ints, of [out_heads, S, 128] bf16 layer
    outputs, on this GPU or mapped from peers) at heads [head_base, head_base + BH).
    Returns the base-2 LSE of these heads (or None)."""
    _check_attention_inputs(q3, k3, v3, ids, logw, text_k, text_v)
    bh, seq, _ = q3.shape
    samples = ids.shape[-1]
    text_tokens = 0 if text_k is None else text_k.shape[1]
    lse_ = torch.empty((bh, seq), dtype=torch.float32, device=q3.device) if return_lse else None
    ws = prefill_workspace(bh, seq, samples, text_tokens, q3.device)
    if ws is None:
        raise RuntimeError("this shape cannot take the paired prefill, so it cannot scatter")
    ptrs = (ctypes.c_void_p * len(outs))(*[int(p) for p in outs])
    lib = _lib.load()
    with torch.cuda.device(q3.device):
        _lib.check(lib.abx_sparse_prefill_scatter(
            _lib.ptr(q3), _lib.ptr(k3), _lib.ptr(v3), bh, seq, _lib.ptr(ids), _lib.ptr(logw), samples,
            _lib.ptr(text_k), _lib.ptr(text_v), text_tokens, ptrs, len(outs), head_base, out_heads, _lib.ptr(lse_),
            _lib.ptr(ws), ws.numel(), _lib.stream_of(q3)), "abx_sparse_prefill_scatter")
    return lse_


def dense_prefill(q3, k3, v3, *, return_lse=False):
    """Dense attention through the same prefill kernel (the dense comparator)."""
    _check_attention_inputs(q3, k3, v3)
    bh, seq, _ = q3.shape
    o = torch.empty_like(q3)
    lse_ = torch.empty((bh, seq), dtype=torch.float32, device=q3.device) if return_lse else None
    lib = _lib.load()
    with torch.cuda.device(q3.device):
        _lib.check(lib.abx_dense_prefill(_lib.ptr(q3), _lib.ptr(k3), _lib.ptr(v3), bh, seq, _lib.ptr(o),
                                         _lib.ptr(lse_), _lib.stream_of(q3)), "abx_dense_prefill")
    return o, lse_


def cross_prefill(q3, k3, v3, *, ids=None, logw=None, samples=0, text_k=None, text_v=None, return_lse=False):
    """q3 [BH,Nq,128] over `samples` granules of k3/v3 [BH,Nk,128] (the plan's ids
    with their log weights, or the first `samples` in order when ids is None)
    followed by every key of text_k/text_v [BH,T,128] (any T)."""
    kv_tokens = 0 if k3 is None else k3.shape[1]
    if text_k is not None and text_v is not None and text_k.ndim == 3 and text_k.shape[1] == 0 \
            and text_v.shape == text_k.shape:
        text_k = text_v = None  # an empty prompt adds no keys
    if ids is not None and ids.ndim == 2 and ids.shape[1] != samples:
        raise RuntimeError(f"samples ({samples}) must equal the ids' column count ({ids.shape[1]})")
    _check_attention_inputs(q3, k3, v3, ids, logw, text_k, text_v, kv_tokens=kv_tokens)
    bh, q_tokens, _ = q3.shape
    o = torch.empty_like(q3)
    lse_ = torch.empty((bh, q_tokens), dtype=torch.float32, device=q3.device) if return_lse else None
    text_tokens = 0 if text_k is None else text_k.shape[1]
    lib = _lib.load()
    with torch.cuda.device(q3.device):
        _lib.check(lib.abx_cross_prefill(_lib.ptr(q3), q_tokens, _lib.ptr(k3), _lib.ptr(v3), kv_tokens, bh,
                                         _lib.ptr(ids), _lib.ptr(logw), samples, _lib.ptr(text_k), _lib.ptr(text_v),
                                         text_tokens, _lib.ptr(o), _lib.ptr(lse_), _lib.stream_of(q3)),
                   "abx_cross_prefill")
    return o, lse_

# ---- torch.library operators ----------------------------------------------------------
# `torch.ops.ab_attention.{ibcs, sip, build_plan, sparse_prefill}`: C++ operators
# (csrc/torch_ops.cpp, TORCH_LIBRARY over the same C ABI) with CUDA and Meta
# kernels only. A CPU tensor finds no kernel and raises, so there is no silent
# fallback; C++ and TorchScript callers reach them without Python.

def _load_torch_ops() -> bool:
    """Registers the operators when libabx_torch.so is built. Before the build
    (the build itself imports this package) they are simply absent, like every
    kernel entry point, which raises until libabx.so exists."""
    path = _lib.PKG / "libabx_torch.so"
    if not path.exists():
        return False
    torch.ops.load_library(str(path))
    return True


TORCH_OPS_LOADED = _load_torch_ops()
