"""``triton_llm.ops.flash_attention`` (reference: python/triton_llm/ops/flash_attention.py), the sm_100a kernel."""
from tritonllmcompiler_b200.ops.flash_attention import flash_attention

__all__ = ["flash_attention"]
