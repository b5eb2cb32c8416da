"""Shared test helpers: golden fixtures and tensor conversions."""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np

from tests.golden.make_golden import CASES, bf16_bits_to_f32, inputs, sip_edge_scores  # noqa: F401

GOLDEN = Path(__file__).resolve().parent / "golden"


def golden(name: str):
    return np.load(GOLDEN / f"{name}.npz")


def case_dims(case: str):
    bh, (t, h, w), _, samples, _ = CASES[case]
    tokens = t * h * w
    return bh, tokens, math.ceil(tokens / 128), tokens // 4, samples


def to_device_bf16(bits: np.ndarray, device="cuda"):
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(device).view(torch.bfloat16)


def bf16_bits(t) -> np.ndarray:
    import torch

    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def f16_bits(t) -> np.ndarray:
    import torch

    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
