"""``triton_llm.ops.swiglu`` (reference: python/triton_llm/ops/swiglu.py), the sm_100a kernel."""
from tritonllmcompiler_b200.ops.swiglu import swiglu

__all__ = ["swiglu"]
