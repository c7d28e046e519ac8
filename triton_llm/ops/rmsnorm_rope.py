"""``triton_llm.ops.rmsnorm_rope`` (reference: python/triton_llm/ops/rmsnorm_rope.py), the sm_100a kernel."""
from tritonllmcompiler_b200.ops.rmsnorm_rope import rmsnorm_rope

__all__ = ["rmsnorm_rope"]
