"""B200-native (sm_100a) drop-in for the ``triton_llm`` operator package.

Exports the same four operators as ``triton_llm`` (python/triton_llm/__init__.py:2-8):
``flash_attention``, ``paged_attention``, ``rmsnorm_rope`` and ``swiglu``, each a thin
PyTorch wrapper over hand-written CUDA in ``libtllm_sm100a.so``.
"""
from tritonllmcompiler_b200.ops.flash_attention import flash_attention
from tritonllmcompiler_b200.ops.paged_attention import paged_attention
from tritonllmcompiler_b200.ops.rmsnorm_rope import rmsnorm_rope
from tritonllmcompiler_b200.ops.swiglu import swiglu

__all__ = ["flash_attention", "paged_attention", "rmsnorm_rope", "swiglu"]
__version__ = "0.2.0"
