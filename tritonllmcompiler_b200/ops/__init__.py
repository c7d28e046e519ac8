"""Device operators. Import the op you need; the package root re-exports them.

Same module layout and names as ``triton_llm.ops`` (python/triton_llm/ops/__init__.py:2-7).
"""
from tritonllmcompiler_b200.ops.flash_attention import flash_attention
from tritonllmcompiler_b200.ops.paged_attention import paged_attention
from tritonllmcompiler_b200.ops.rmsnorm_rope import rmsnorm_rope
from tritonllmcompiler_b200.ops.swiglu import swiglu

__all__ = ["flash_attention", "paged_attention", "rmsnorm_rope", "swiglu"]
