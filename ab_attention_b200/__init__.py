"""B200-native AB-Attention sparse-attention hot path (IBCS + SIP + HT-weighted sparse prefill)."""
from .attention import (SamplePlan, ab_attention, apply_plan, build_plan, dense_attention,
                        dense_cross_attention, paged_attention)
from .layout import cube_layout

__all__ = ["SamplePlan", "ab_attention", "apply_plan", "build_plan", "dense_attention", "dense_cross_attention",
           "paged_attention", "cube_layout", "VideoAttention", "hunyuan_attention", "ab_attention_host"]
from .video import VideoAttention, hunyuan_attention  # noqa: E402
from .pipeline import ab_attention_host  # noqa: E402
