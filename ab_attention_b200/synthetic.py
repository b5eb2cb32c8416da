"""Seeded synthetic video-token Q/K/V at the benchmark shapes.

Model activations and the prompt benchmark behind the reference's quality
numbers are not available, so the benchmark configurations use a smooth
random field over token positions instead:

    Q, K per head = A . phi(t, h, w) + 0.3 * eps,   V ~ N(0, 1)

phi = 16 random Fourier features cos(w_f . (t, h, w) + b_f) with frequencies
w_f ~ N(0, sigma^2) per axis (sigma = 0.1 unless swept) and phases b_f ~ U(0,
2 pi), shared by all heads; A ~ N(0, 1/4) of shape [D, 16] per (batch, head),
shared by Q and K of that head; eps ~ N(0, 1) drawn separately for Q and K.
Tokens are row-major (t, h, w).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class VideoShape:
    name: str
    batch: int
    heads: int
    frames: int
    height: int
    width: int
    sample_pages: int
    seed: int
    text_tokens: int = 0
    sigma: float = 0.1
    cube: bool = False
    dim: int = 128
    extra: dict = field(default_factory=dict, compare=False, hash=False)

    @property
    def tokens(self) -> int:
        return self.frames * self.height * self.width

    @property
    def batch_heads(self) -> int:
        return self.batch * self.heads


# BASELINE configurations 1-4 (configuration 0 is the CPU-only D=64 case).
CONFIGS = {
    "wan1.3b": VideoShape("wan1.3b", 1, 12, 21, 45, 80, 64, 1),
    "wan14b": VideoShape("wan14b", 2, 40, 21, 45, 80, 64, 2),
    "hunyuan13b": VideoShape("hunyuan13b", 1, 24, 33, 45, 80, 71, 3, text_tokens=256),
    "wan14b-cube": VideoShape("wan14b-cube", 1, 40, 21, 45, 80, 64, 4, cube=True),
}


# the CPU plumbing case, run through the reference math
# in PyTorch on the host only (D = 64 and fp32 are outside the kernels' contract;
# "2 deterministic + 6 sampled pages" is sample_pages = 8, the pi = 1 units coming
# out of the certainty loop as in the reference).
CPU_PLUMBING = VideoShape("cpu-plumbing", 1, 2, 4, 32, 32, 8, 0, dim=64)


def smooth_field(batch_heads: int, frames: int, height: int, width: int, *, dim: int = 128,
                 seed: int = 0, sigma: float = 0.1, device="cuda", dtype=torch.bfloat16,
                 features: int = 16, heads: range | None = None):
    """Return (q, k, v) of shape [len(heads), frames*height*width, dim].

    Each head draws from its own generator (seeded by (seed, head)), so any
    subset of heads, e.g. one GPU's shard, is identical to the same heads of
    the full tensor.
    """
    heads = range(batch_heads) if heads is None else heads
    gen = torch.Generator(device=device).manual_seed(seed)
    tokens = frames * height * width
    freq = torch.randn(features, 3, generator=gen, device=device) * sigma
    phase = torch.rand(features, generator=gen, device=device) * (2 * torch.pi)
    t = torch.arange(frames, device=device, dtype=torch.float32)
    h = torch.arange(height, device=device, dtype=torch.float32)
    w = torch.arange(width, device=device, dtype=torch.float32)
    pos = torch.stack(torch.meshgrid(t, h, w, indexing="ij"), dim=-1).reshape(tokens, 3)
    phi = torch.cos(pos @ freq.T + phase)  # [tokens, features]
    q = torch.empty(len(heads), tokens, dim, dtype=dtype, device=device)
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    for i, head in enumerate(heads):
        hg = torch.Generator(device=device).manual_seed(seed * 1_000_003 + head + 1)
        a = torch.randn(dim, features, generator=hg, device=device) * 0.5
        field_ = phi @ a.T  # [tokens, dim]
        q[i] = (field_ + 0.3 * torch.randn(tokens, dim, generator=hg, device=device)).to(dtype)
        k[i] = (field_ + 0.3 * torch.randn(tokens, dim, generator=hg, device=device)).to(dtype)
        v[i] = torch.randn(tokens, dim, generator=hg, device=device).to(dtype)
    return q, k, v


def make_inputs(shape: VideoShape, device="cuda", bh_slice: slice | list | None = None):
    """Q/K/V [B, H, N, 128] for a configuration (cube-permuted when shape.cube),
    plus (text_k, text_v) [B, H, 256, 128] when the configuration has text.
    `bh_slice` (a slice or a list of flattened heads) selects heads; the result
    is then [1, len, N, 128]."""
    if bh_slice is None:
        heads = range(shape.batch_heads)
    elif isinstance(bh_slice, slice):
        heads = range(shape.batch_heads)[bh_slice]
    else:
        heads = list(bh_slice)
    q, k, v = smooth_field(shape.batch_heads, shape.frames, shape.height, shape.width, dim=shape.dim,
                           seed=shape.seed, sigma=shape.sigma, device=device, heads=heads)
    if shape.cube:
        from .layout import cube_layout

        order, _ = cube_layout(shape.frames, shape.height, shape.width, device=device)
        q, k, v = (x.index_select(1, order) for x in (q, k, v))
    if bh_slice is not None:
        shape4 = (1, q.shape[0], shape.tokens, shape.dim)
    else:
        shape4 = (shape.batch, shape.heads, shape.tokens, shape.dim)
    q, k, v = (x.reshape(shape4) for x in (q, k, v))
    text = None
    if shape.text_tokens:
        gen = torch.Generator(device=device).manual_seed(shape.seed + 7919)
        tk = torch.randn(shape.batch_heads, shape.text_tokens, shape.dim, generator=gen, device=device)
        tv = torch.randn(shape.batch_heads, shape.text_tokens, shape.dim, generator=gen, device=device)
        if bh_slice is not None:
            tk, tv = tk[bh_slice], tv[bh_slice]
        text = tuple(x.to(torch.bfloat16).reshape(shape4[0], shape4[1], -1, shape.dim).contiguous()
                     for x in (tk, tv))
    return q, k, v, text
