"""Denoising schedule with per-layer sample-plan reuse (ab_attention/video.py:53-87).

The paper schedule keeps the first 10 steps and layer 0 dense; every other layer
builds a fresh plan on steps 11, 15, ..., 47 (an "anchor" every 4 steps) and
reuses it on the steps in between. `VideoAttention` keeps the reference's API
(`reset`, `step_end` as Diffusers' `callback_on_step_end`, `is_sparse`,
`attend`), anchors and seeds, so its plans are bit-identical to the reference's.
A B200 holds the plans in device memory (the reference parks them in pinned
host RAM to fit a single 80 GB GPU): a Wan2.1-14B layer's plan is 0.39 GB.
"""
from __future__ import annotations

import torch

from .attention import SamplePlan, apply_plan, build_plan, dense_attention, dense_cross_attention


def plan_seed(layer: int, anchor: int) -> int:
    """Seed of the plan a layer builds at an anchor step (ab_attention/video.py:79)."""
    return 42 + layer * 1_000_003 + anchor * 97


def anchor_step(step: int) -> int:
    """The refresh step a sparse step reuses the plan of (ab_attention/video.py:77)."""
    return 11 + (step - 11) // 4 * 4


class VideoAttention:
    """One pipeline's denoising schedule and per-layer sample plans.

    Call ``reset()`` before each video and pass ``step_end`` as Diffusers'
    ``callback_on_step_end``. Wan's two sequential CFG calls share one plan.
    ``host_plans=True`` keeps stored plans in pinned host memory as the
    reference does (for callers short of device memory).
    """

    def __init__(self, sample_pages, *, dense=False, host_plans=False):
        self.sample_pages = sample_pages
        self.dense = dense
        self.host_plans = host_plans
        self.reset()

    def reset(self):
        self.step = 1
        self.plans = {}

    def step_end(self, pipe, index, timestep, callback_kwargs):
        self.step = index + 2  # Diffusers indices are zero-based.
        return callback_kwargs

    def is_sparse(self, layer):
        return not self.dense and self.step > 10 and layer > 0

    def _store(self, plan: SamplePlan, previous: SamplePlan | None) -> SamplePlan:
        if not self.host_plans:
            return plan
        if previous is None:
            previous = SamplePlan(*(torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in plan))
        for storage, tensor in zip(previous, plan):
            storage.copy_(tensor)
        return previous

    def attend(self, layer, q, k, v, *, return_lse=False, text_kv=None):
        """Sparse attention of one layer at the current step, building the plan
        on an anchor step and reusing it otherwise."""
        anchor = anchor_step(self.step)
        stored_anchor, stored = self.plans.get(layer, (None, None))
        if stored_anchor != anchor:
            plan = build_plan(q, k, sample_pages=self.sample_pages, seed=plan_seed(layer, anchor))
            self.plans[layer] = (anchor, self._store(plan, stored))
        else:
            plan = SamplePlan(*(t.to(q.device, non_blocking=True) for t in stored))
        return apply_plan(q, k, v, plan, return_lse=return_lse, text_kv=text_kv)

    def __call__(self, layer, q, k, v, *, return_lse=False, text_kv=None):
        """Dense on the steps and layer the schedule keeps dense, else `attend`."""
        if self.is_sparse(layer):
            return self.attend(layer, q, k, v, return_lse=return_lse, text_kv=text_kv)
        if text_kv is not None:
            raise ValueError("text keys are only supported on sparse steps")
        return dense_attention(q, k, v, return_lse=return_lse)


def hunyuan_attention(schedule, layer, q, k, v, video_tokens, prompt_tokens):
    """One HunyuanVideo attention layer over [video | prompt | padding] tokens
    (ab_attention/video.py:129-151).

    On sparse steps the video queries attend to the layer's sampled video keys
    plus every prompt key with weight pi = 1 (the reference merges a sparse
    video state with an exact video->text state by LSE; that is the same
    softmax over the union, here one kernel), and the prompt queries attend
    exactly to every video and prompt key. On dense steps the video and prompt
    tokens attend exactly to each other. Padding tokens always form their own
    exact partition. q, k, v: [B, H, N, 128] bf16.
    """
    prompt_end = video_tokens + prompt_tokens
    sl = lambda x, a, b: x[:, :, a:b].contiguous()  # noqa: E731
    text_kv = (sl(k, video_tokens, prompt_end), sl(v, video_tokens, prompt_end)) if prompt_tokens else None
    video_k, video_v = sl(k, 0, video_tokens), sl(v, 0, video_tokens)
    if schedule.is_sparse(layer):
        outputs = [schedule.attend(layer, sl(q, 0, video_tokens), video_k, video_v, text_kv=text_kv)]
        if prompt_tokens:
            outputs.append(dense_cross_attention(sl(q, video_tokens, prompt_end), video_k, video_v,
                                                 extra_kv=text_kv))
    else:
        outputs = [dense_cross_attention(sl(q, 0, prompt_end), video_k, video_v, extra_kv=text_kv)]
    if prompt_end < q.shape[2]:
        outputs.append(dense_cross_attention(sl(q, prompt_end, q.shape[2]), None, None,
                                             extra_kv=(sl(k, prompt_end, q.shape[2]), sl(v, prompt_end, q.shape[2]))))
    return torch.cat(outputs, dim=2)
