"""Stand-in for the reference's compiled module `ab_attention._C`
(csrc/bindings.cpp:3-8, csrc/ops.h:5-8): the same two calls with the same
argument meaning, backed by the C++ operators torch.ops.ab_attention (CUDA only).

    ibcs(q, k) -> scores f32 [B*H*ceil(S/128), S/4]        (q, k: bf16 [B, H, S, 128])
    sip(scores, offsets, ids, logs) -> None               (ids/logs written in place)
"""
import torch

import ab_attention_b200.ops  # noqa: F401  (loads the operator library)


def ibcs(q: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    return torch.ops.ab_attention.ibcs(q, k)


def sip(scores: torch.Tensor, offsets: torch.Tensor, ids: torch.Tensor, logs: torch.Tensor) -> None:
    torch.ops.ab_attention.sip(scores, offsets, ids, logs)
