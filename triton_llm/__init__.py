"""The ``triton_llm`` import name, served by the B200 (sm_100a) kernels.

Callers of the reference package keep their import lines unchanged
(``import triton_llm``, ``from triton_llm.ops.swiglu import swiglu``; the reference's
python/triton_llm/__init__.py:2-8): the four operators resolve to the hand-written CUDA in
``tritonllmcompiler_b200``. Only the operator surface is provided; the reference's
``triton_llm.reference`` oracles, compiler tooling and tile-policy tables are not part of it.
"""
from triton_llm.ops.flash_attention import flash_attention
from triton_llm.ops.paged_attention import paged_attention
from triton_llm.ops.rmsnorm_rope import rmsnorm_rope
from triton_llm.ops.swiglu import swiglu

__all__ = ["flash_attention", "paged_attention", "rmsnorm_rope", "swiglu"]
__version__ = "0.2.0"
