"""``triton_llm.ops.paged_attention`` (reference: python/triton_llm/ops/paged_attention.py), the sm_100a kernel."""
from tritonllmcompiler_b200.ops.paged_attention import paged_attention

__all__ = ["paged_attention"]
