"""CPU oracle for the AB-Attention hot path (test infrastructure only).

ORACLE INFRASTRUCTURE: only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg import this module, and only as the checker. The shipped
package (ab_attention_b200) never imports it.

* IBCS / SIP: ctypes wrapper over oracle/abx_oracle.c (a scalar C restatement of
  csrc/ibcs.cu and csrc/sip.cu; see the header of that file).
* Prefill: a float64 numpy evaluation of the sampled Horvitz-Thompson estimator
  that the reference runs through FlashInfer (ab_attention/flashinfer_backend.py:
  30-58 transform + OnlineSoftmax; keys of slot s are tokens 4*ids[s] + 0..3,
  logit l = (q.k) * 128^-0.5 * log2(e) + log_weights[s], o = softmax_2(l) V,
  lse = log2 sum 2^l).
* Cube layout permutation (ab_attention/video.py:97-105).
"""
from __future__ import annotations

import ctypes
import math
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"
KAPPA = np.float32(128 ** -0.5 * 1.4426950408889634)

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        _lib = ctypes.CDLL(str(LIB))
        p = ctypes.c_void_p
        i64 = ctypes.c_int64
        _lib.oracle_cluster.argtypes = [p, i64, i64, p, p, p, p]
        _lib.oracle_pool.argtypes = [p, i64, i64, p]
        _lib.oracle_lse.argtypes = [p, p, i64, i64, i64, ctypes.c_float, p, p, p]
        _lib.oracle_mix.argtypes = [p, p, p, p, i64, i64, p]
        _lib.oracle_sip.argtypes = [p, p, i64, ctypes.c_int, p, p, ctypes.c_int]
    return _lib


def _ptr(a: np.ndarray):
    assert a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.c_void_p)


# ---- bf16 helpers (numpy has no bfloat16) ----------------------------------

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))
    return (rounded >> 16).astype(np.uint16)


# ---- IBCS / SIP ------------------------------------------------------------

def cluster(q_bits: np.ndarray, with_quotient: bool = False):
    """q_bits: uint16 bf16 [bh, seq, 128] -> (centroid bits [rows,8,128], populations [rows,8],
    assignments [rows,128]) and, with_quotient, the float centroids before bf16 rounding."""
    bh, seq, _ = q_bits.shape
    qb = math.ceil(seq / 128)
    cent = np.zeros((bh * qb, 8, 128), np.uint16)
    pops = np.zeros((bh * qb, 8), np.float32)
    assign = np.zeros((bh * qb, 128), np.int32)
    quot = np.zeros((bh * qb, 8, 128), np.float32)
    q_bits = np.ascontiguousarray(q_bits)
    lib().oracle_cluster(_ptr(q_bits), bh, seq, _ptr(cent), _ptr(pops), _ptr(assign), _ptr(quot))
    return (cent, pops, assign, quot) if with_quotient else (cent, pops, assign)


def pool(k_bits: np.ndarray) -> np.ndarray:
    bh, seq, _ = k_bits.shape
    out = np.zeros((bh, seq // 4, 2, 128), np.uint16)
    k_bits = np.ascontiguousarray(k_bits)
    lib().oracle_pool(_ptr(k_bits), bh, seq, _ptr(out))
    return out


def lse(centroid_bits: np.ndarray, pooled_bits: np.ndarray, bh: int, qb: int):
    fine = pooled_bits.shape[1]
    rows = bh * qb
    out = np.zeros((rows, 8, fine), np.uint16)
    mx = np.zeros((rows, 8), np.float32)
    den = np.zeros((rows, 8), np.float32)
    c = np.ascontiguousarray(centroid_bits)
    p = np.ascontiguousarray(pooled_bits)
    lib().oracle_lse(_ptr(c), _ptr(p), bh, qb, fine, KAPPA, _ptr(out), _ptr(mx), _ptr(den))
    return out, mx, den


def mix(lse_bits: np.ndarray, populations, lse_max, lse_den) -> np.ndarray:
    rows, _, fine = lse_bits.shape
    out = np.zeros((rows, fine), np.float32)
    args = [np.ascontiguousarray(a) for a in (lse_bits, populations.astype(np.float32), lse_max, lse_den)]
    lib().oracle_mix(*map(_ptr, args), rows, fine, _ptr(out))
    return out


def ibcs(q_bits: np.ndarray, k_bits: np.ndarray) -> np.ndarray:
    """Full IBCS: bf16 bits q/k [bh, seq, 128] -> scores [rows, seq/4]."""
    bh, seq, _ = q_bits.shape
    qb = math.ceil(seq / 128)
    cent, pops, _ = cluster(q_bits)
    pooled = pool(k_bits)
    l, mx, den = lse(cent, pooled, bh, qb)
    return mix(l, pops, mx, den)


def sip(scores: np.ndarray, offsets: np.ndarray, samples: int):
    rows, population = scores.shape
    ids = np.zeros((rows, samples), np.int32)
    logw = np.zeros((rows, samples), np.float32)
    s = np.ascontiguousarray(scores, dtype=np.float32)
    o = np.ascontiguousarray(offsets, dtype=np.float32)
    lib().oracle_sip(_ptr(s), _ptr(o), rows, population, _ptr(ids), _ptr(logw), samples)
    return ids, logw


# ---- prefill -----------------------------------------------------------------

def prefill_row(qh, kh, vh, row_ids, row_weights, r, text_k=None, text_v=None):
    """One plan row (query block r of one head) of the float64 HT estimator:
    keys are tokens 4*id + 0..3 of the row's granules, each with logit shift
    log_weights[slot] (flashinfer_backend.py:30-58), followed by the always-
    included text keys (shift 0); logits scaled by D^-1/2 * log2(e) (D = 128 in
    the reference). Returns (o [n, D], lse [n]) for the block's n = min(128,
    seq - 128 r) queries."""
    kappa = qh.shape[-1] ** -0.5 * math.log2(math.e)
    tok = (4 * np.asarray(row_ids, dtype=np.int64)[:, None] + np.arange(4)[None, :]).reshape(-1)
    keys = np.asarray(kh[tok], dtype=np.float64)
    vals = np.asarray(vh[tok], dtype=np.float64)
    w = np.repeat(np.asarray(row_weights, dtype=np.float64), 4)
    if text_k is not None:
        keys = np.concatenate([keys, np.asarray(text_k, dtype=np.float64)])
        vals = np.concatenate([vals, np.asarray(text_v, dtype=np.float64)])
        w = np.concatenate([w, np.zeros(len(text_k))])
    qs = np.asarray(qh[r * 128:(r + 1) * 128], dtype=np.float64)
    logits = qs @ keys.T * kappa + w[None, :]
    m = logits.max(axis=1, keepdims=True)
    p = np.exp2(logits - m)
    s = p.sum(axis=1, keepdims=True)
    return (p @ vals) / s, (m + np.log2(s))[:, 0]


def prefill(q, k, v, ids, log_weights, text_k=None, text_v=None):
    """Float64 evaluation of the HT-weighted sparse prefill.

    q/k/v: float arrays [bh, seq, 128] (already rounded to bf16 values);
    ids/log_weights: [rows, samples] (rows = bh * ceil(seq/128));
    text_k/text_v: optional [bh, T, 128] always-included keys with weight 0.
    Returns (o [bh, seq, 128] float64, lse [bh, seq] float64, base 2).
    """
    bh, seq, dim = q.shape
    qb = math.ceil(seq / 128)
    o = np.zeros((bh, seq, dim))
    lse = np.zeros((bh, seq))
    for h in range(bh):
        qh = np.asarray(q[h], dtype=np.float64)
        kh = np.asarray(k[h], dtype=np.float64)
        vh = np.asarray(v[h], dtype=np.float64)
        for r in range(qb):
            row = h * qb + r
            oo, ll = prefill_row(qh, kh, vh, ids[row], log_weights[row], r,
                                 None if text_k is None else text_k[h], None if text_v is None else text_v[h])
            o[h, r * 128:r * 128 + len(oo)] = oo
            lse[h, r * 128:r * 128 + len(oo)] = ll
    return o, lse


def dense(q, k, v):
    """Float64 dense softmax attention with 128^-0.5 scaling; lse in base 2."""
    bh, seq, _ = q.shape
    o = np.zeros(q.shape)
    lse = np.zeros((bh, seq))
    kappa = 128 ** -0.5 * math.log2(math.e)
    for h in range(bh):
        logits = q[h].astype(np.float64) @ k[h].astype(np.float64).T * kappa
        m = logits.max(axis=1, keepdims=True)
        p = np.exp2(logits - m)
        s = p.sum(axis=1, keepdims=True)
        o[h] = p @ v[h].astype(np.float64) / s
        lse[h] = (m + np.log2(s))[:, 0]
    return o, lse


def cube_order(t: int, h: int, w: int) -> np.ndarray:
    """4x4x4 cube permutation of a row-major (t,h,w) token grid; boundary cubes
    keep only their valid tokens (ab_attention/video.py:97-105)."""
    grid = np.arange(t * h * w).reshape(t, h, w)
    pt, ph, pw = -t % 4, -h % 4, -w % 4
    grid = np.pad(grid, ((0, pt), (0, ph), (0, pw)), constant_values=-1)
    nt, nh, nw = (s // 4 for s in grid.shape)
    order = grid.reshape(nt, 4, nh, 4, nw, 4).transpose(0, 2, 4, 1, 3, 5).reshape(-1)
    return order[order >= 0]
