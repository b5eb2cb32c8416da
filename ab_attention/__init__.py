"""`ab_attention` import name for the B200 build (ab_attention_b200).

Installs under the reference's package name so existing callers keep their
imports: `from ab_attention import build_plan, apply_plan, ab_attention,
SamplePlan` (ab_attention/__init__.py:1-3 of the reference), `from
ab_attention.attention import ...` (what the reference's video.py:10 imports),
`ab_attention._C` (the native `ibcs` / `sip` ops, csrc/bindings.cpp:3-8) and
`ab_attention.flashinfer_backend.paged_attention` (flashinfer_backend.py:164-242)
all resolve to the sm_100a implementation.
"""
from ab_attention_b200.attention import SamplePlan, ab_attention, apply_plan, build_plan

__all__ = ["SamplePlan", "ab_attention", "apply_plan", "build_plan"]
