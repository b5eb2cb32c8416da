"""`ab_attention.flashinfer_backend.paged_attention` (reference
flashinfer_backend.py:164-242): same signature, checks and outputs, served by the
tcgen05 sparse prefill instead of FlashInfer's fa3 backend."""
from ab_attention_b200.attention import paged_attention  # noqa: F401
