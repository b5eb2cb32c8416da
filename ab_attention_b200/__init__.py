"""B200-native AB-Attention sparse-attention hot path (IBCS + SIP + HT-weighted sparse prefill)."""
from .attention import SamplePlan, ab_attention, apply_plan, build_plan, dense_attention
from .layout import cube_layout

__all__ = ["SamplePlan", "ab_attention", "apply_plan", "build_plan", "dense_attention", "cube_layout"]
