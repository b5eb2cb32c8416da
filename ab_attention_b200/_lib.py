"""ctypes binding of libabx.so (the C ABI declared in include/abx.h).

There is no CPU fallback: if the library is missing or no CUDA device is
present, calls raise. Torch tensors are passed as raw device pointers on the
caller's current CUDA stream.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libabx.so"
HEADER = PKG.parent / "include" / "abx.h"

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_SIGNATURES = {
    "abx_version": ([], ctypes.c_int),
    "abx_status_string": ([ctypes.c_int], ctypes.c_char_p),
    "abx_last_error": ([], ctypes.c_char_p),
    "abx_device_status": ([_p, ctypes.c_int, _p], ctypes.c_int),
    "abx_selftest_wait_timeout": ([_i64, _p], ctypes.c_int),
    "abx_ibcs_cluster": ([_p, _i64, _i64, _p, _p, _p, _p, _p], ctypes.c_int),
    "abx_ibcs_pool": ([_p, _i64, _i64, _p, _p], ctypes.c_int),
    "abx_ibcs_lse": ([_p, _p, _i64, _i64, _i64, _p, _p, _p, _p], ctypes.c_int),
    "abx_ibcs_mix": ([_p, _p, _p, _p, _i64, _i64, _p, _p], ctypes.c_int),
    "abx_ibcs_workspace_size": ([_i64, _i64, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "abx_ibcs_scores": ([_p, _p, _i64, _i64, _p, _p, ctypes.c_size_t, _p], ctypes.c_int),
    "abx_sip": ([_p, _p, _i64, _i64, _p, _p, _i64, _p], ctypes.c_int),
    "abx_build_plan": ([_p, _p, _i64, _i64, _p, _i64, _p, _p, _p, ctypes.c_size_t, _p], ctypes.c_int),
    "abx_static_scratch_bytes": ([], ctypes.c_size_t),
    "abx_build_plan_static": ([_p, _p, _i64, _i64, _p, _i64, _p, _p, _p], ctypes.c_int),
    "abx_sparse_prefill": ([_p, _p, _p, _i64, _i64, _p, _p, _i64, _p, _p, _i64, _p, _p, _p], ctypes.c_int),
    "abx_prefill_workspace_size": ([_i64, _i64, _i64, _i64, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "abx_sparse_prefill_paired": ([_p, _p, _p, _i64, _i64, _p, _p, _i64, _p, _p, _i64, _p, _p, _p, ctypes.c_size_t,
                                   _p], ctypes.c_int),
    "abx_pair_plan": ([_p, _i64, _i64, _i64, _i64, _p, ctypes.c_size_t, _p], ctypes.c_int),
    "abx_sparse_prefill_paired_planned": ([_p, _p, _p, _i64, _i64, _p, _p, _i64, _p, _p, _i64, _p, _p, _p,
                                           ctypes.c_size_t, _p], ctypes.c_int),
    "abx_ipc_handle": ([_p, _p, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "abx_ipc_open": ([_p, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "abx_ipc_close": ([_p], ctypes.c_int),
    "abx_peer_copy": ([_p, _p, ctypes.c_size_t, _p], ctypes.c_int),
    "abx_sparse_prefill_scatter": ([_p, _p, _p, _i64, _i64, _p, _p, _i64, _p, _p, _i64, _p, ctypes.c_int, _i64,
                                    _i64, _p, _p, ctypes.c_size_t, _p], ctypes.c_int),
    "abx_dense_prefill": ([_p, _p, _p, _i64, _i64, _p, _p, _p], ctypes.c_int),
    "abx_cross_prefill": ([_p, _i64, _p, _p, _i64, _i64, _p, _p, _i64, _p, _p, _i64, _p, _p, _p], ctypes.c_int),
}

_lib = None


class AbxError(RuntimeError):
    """A libabx call returned a nonzero status."""


def header_symbols() -> list[str]:
    """Every function name declared in include/abx.h."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(abx_\w+)\s*\(", text, re.M)))


def load():
    """Load libabx.so (no CUDA call is made)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise AbxError(f"{LIB_PATH} is not built; run python -m ab_attention_b200.build")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        lib = load()
        raise AbxError(f"{what} failed: {lib.abx_status_string(status).decode()}: "
                       f"{lib.abx_last_error().decode()}")


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise AbxError("libabx kernels need CUDA tensors (there is no CPU implementation)")


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def device_status(device=None, clear: bool = False) -> int:
    """Sticky device-side error word (0 = none); synchronises the current stream."""
    lib = load()
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    out = ctypes.c_int(0)
    with torch.cuda.device(device):
        s = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        check(lib.abx_device_status(s, int(clear), ctypes.byref(out)), "abx_device_status")
    return out.value
