"""`ab_attention.attention` (reference ab_attention/attention.py:11-102) on B200."""
from ab_attention_b200.attention import (SamplePlan, ab_attention, apply_plan, build_plan,  # noqa: F401
                                         dense_attention, paged_attention)
