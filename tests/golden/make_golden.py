"""Generate the golden vectors in tests/golden/ from the reference's own kernels.

Runs on a GPU box: the reference IBCS/SIP CUDA kernels, compiled from the
reference sources for sm_100a by oracle/build_ref.py (oracle/_ref/abx_ref*.so),
are executed on seeded inputs and every stage output is saved:

    python tests/golden/make_golden.py OUT_DIR

Inputs are produced by `inputs(case)` below from numpy's PCG64 generator, so
the CPU tests regenerate them bit for bit instead of storing them. Do not
change `inputs` or CASES without regenerating the fixtures.
"""
from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]

# name: (batch_heads, (frames, height, width), sigma, samples, seed)
CASES = {
    "g512": (2, (2, 16, 16), 0.1, 32, 11),
    "g1028": (1, (1, 4, 257), 0.2, 64, 12),
    "g2048": (1, (2, 32, 32), 0.3, 96, 13),
}


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def inputs(case: str):
    """Smooth-field q/k and N(0,1) v as bf16 bit patterns [bh, tokens, 128] (uint16)."""
    bh, (t, h, w), sigma, _, seed = CASES[case]
    rng = np.random.Generator(np.random.PCG64(seed))
    freq = rng.standard_normal((16, 3)) * sigma
    phase = rng.uniform(0.0, 2 * np.pi, 16)
    pos = np.stack(np.meshgrid(np.arange(t), np.arange(h), np.arange(w), indexing="ij"), -1).reshape(-1, 3)
    phi = np.cos(pos @ freq.T + phase)
    tokens = t * h * w
    q = np.empty((bh, tokens, 128), np.uint16)
    k = np.empty_like(q)
    v = np.empty_like(q)
    for head in range(bh):
        a = rng.standard_normal((128, 16)) * 0.5
        field = phi @ a.T
        q[head] = f32_to_bf16_bits((field + 0.3 * rng.standard_normal((tokens, 128))).astype(np.float32))
        k[head] = f32_to_bf16_bits((field + 0.3 * rng.standard_normal((tokens, 128))).astype(np.float32))
        v[head] = f32_to_bf16_bits(rng.standard_normal((tokens, 128)).astype(np.float32))
    return q, k, v


def sip_edge_scores():
    """Hand-made SIP rows: uniform, a dominant unit, zeros (clamped), staged certainty, ties."""
    population, rows = 256, 6
    s = np.full((rows, population), 1.0 / population, np.float32)
    s[1, 17] = 0.9
    s[2, :200] = 0.0
    s[3, :10] = np.linspace(0.2, 0.05, 10)
    s[4, ::2] = 0.0
    s[5] = np.repeat(np.float32([0.5, 1e-3, 2.0, 1e-35]), population // 4)
    offsets = np.float32([0.0, 0.5, 0.999, 0.25, 0.75, 0.123])
    return s, offsets


def main(out: Path) -> None:
    import torch

    sys.path.insert(0, str(ROOT))
    from oracle.build_ref import load

    ref = load()
    out.mkdir(parents=True, exist_ok=True)
    dev = torch.device("cuda")
    for case, (bh, _, _, samples, seed) in CASES.items():
        qb_, kb_, _ = inputs(case)
        q = torch.from_numpy(qb_.view(np.int16)).to(dev).view(torch.bfloat16)
        k = torch.from_numpy(kb_.view(np.int16)).to(dev).view(torch.bfloat16)
        tokens = q.shape[1]
        qb = math.ceil(tokens / 128)
        rows = bh * qb
        cent, pops = ref.cluster(q)
        pooled = ref.pool(k)
        lse, mx, den = ref.lse(cent, pooled)
        scores = ref.scores(lse, pops, mx, den)
        scores_full = ref.ibcs(q.unsqueeze(0), k.unsqueeze(0))
        assert torch.equal(scores, scores_full)
        gen = torch.Generator(device=dev).manual_seed(seed)
        offsets = torch.rand(rows, device=dev, generator=gen)
        ids = torch.empty((rows, samples), dtype=torch.int32, device=dev)
        logw = torch.empty((rows, samples), dtype=torch.float32, device=dev)
        ref.sip(scores, offsets, ids, logw)
        torch.cuda.synchronize()
        np.savez_compressed(
            out / f"{case}.npz",
            centroids=cent.view(torch.int16).cpu().numpy().view(np.uint16).reshape(rows, 8, 128),
            populations=pops.float().cpu().numpy().reshape(rows, 8),
            lse=lse.view(torch.int16).cpu().numpy().view(np.uint16),
            lse_max=mx.cpu().numpy(), lse_den=den.cpu().numpy(),
            scores=scores.cpu().numpy(), offsets=offsets.cpu().numpy(),
            ids=ids.cpu().numpy(), log_weights=logw.cpu().numpy())
        print(case, "rows", rows, "F", tokens // 4, "samples", samples)
    s, offsets = sip_edge_scores()
    st = torch.from_numpy(s).to(dev)
    ot = torch.from_numpy(offsets).to(dev)
    for samples in (8, 64, 200):
        ids = torch.empty((s.shape[0], samples), dtype=torch.int32, device=dev)
        logw = torch.empty((s.shape[0], samples), dtype=torch.float32, device=dev)
        ref.sip(st, ot, ids, logw)
        torch.cuda.synchronize()
        np.savez_compressed(out / f"sip_edge_m{samples}.npz", ids=ids.cpu().numpy(), log_weights=logw.cpu().numpy())
        print("sip_edge", samples)


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent)
