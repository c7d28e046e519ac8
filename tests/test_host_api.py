"""Host-side behaviour of the operator wrappers that needs no GPU.

The wrappers keep the reference's signatures and its AssertionError checks
(python/triton_llm/ops/*.py); CPU tensors fail the ``is_cuda`` assert before any launch.
"""
import inspect

import pytest
import torch

import tritonllmcompiler_b200 as pkg
from tritonllmcompiler_b200 import ops


def test_public_surface_matches_reference():
    assert pkg.__all__ == ["flash_attention", "paged_attention", "rmsnorm_rope", "swiglu"]
    assert ops.__all__ == pkg.__all__
    assert pkg.__version__ == "0.2.0"


def test_signatures_match_reference():
    sig = inspect.signature(pkg.flash_attention)
    assert list(sig.parameters) == ["q", "k", "v", "causal", "sm_scale"]
    assert sig.parameters["causal"].kind is inspect.Parameter.KEYWORD_ONLY
    assert sig.parameters["causal"].default is False
    assert sig.parameters["sm_scale"].default is None
    sig = inspect.signature(pkg.paged_attention)
    assert list(sig.parameters) == ["q", "k_cache", "v_cache", "block_tables", "context_lens",
                                    "block_size", "sm_scale"]
    assert sig.parameters["block_size"].kind is inspect.Parameter.KEYWORD_ONLY
    assert sig.parameters["block_size"].default is inspect.Parameter.empty
    sig = inspect.signature(pkg.rmsnorm_rope)
    assert list(sig.parameters) == ["x", "weight", "cos", "sin", "eps"]
    assert sig.parameters["eps"].default == 1e-6
    sig = inspect.signature(pkg.swiglu)
    assert list(sig.parameters) == ["x", "w1", "w3"]


def test_cpu_tensors_are_rejected_like_the_reference():
    q = torch.zeros(1, 1, 8, 64, dtype=torch.float16)
    with pytest.raises(AssertionError):
        pkg.flash_attention(q, q, q)
    with pytest.raises(AssertionError):
        pkg.paged_attention(q[:, :, :1], q, q, torch.zeros(1, 1, dtype=torch.int32),
                            torch.ones(1, dtype=torch.int32), block_size=16)
    x = torch.zeros(1, 2, 1, 64, dtype=torch.float16)
    with pytest.raises(AssertionError):
        pkg.rmsnorm_rope(x, torch.ones(64), torch.ones(2, 64), torch.ones(2, 64))
    with pytest.raises(AssertionError):
        pkg.swiglu(torch.zeros(4, 4), torch.zeros(4, 4), torch.zeros(4, 4))


def test_no_cpu_fallback_in_product_code():
    """The package never imports the oracle or any CPU implementation of the ops."""
    import os

    root = os.path.dirname(pkg.__file__)
    for dirpath, _, files in os.walk(root):
        for f in files:
            if f.endswith(".py"):
                src = open(os.path.join(dirpath, f)).read()
                assert "from oracle" not in src and "import oracle" not in src


def test_host_pipeline_column_blocks():
    from tritonllmcompiler_b200.ops.host_pipeline import _blocks
    for n, c in [(14336, 8), (1000, 3), (128, 8), (100, 4), (14336, 1), (5000, 16)]:
        b = _blocks(n, c)
        assert b[0][0] == 0 and b[-1][1] == n
        assert all(b0 < b1 for b0, b1 in b) and all(b[i][1] == b[i + 1][0] for i in range(len(b) - 1))
        assert all(b0 % 128 == 0 for b0, _ in b) and len(b) <= max(c, 1)
