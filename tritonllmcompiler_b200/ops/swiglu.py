"""SwiGLU dual GEMM on B200: drop-in for ``triton_llm.ops.swiglu``.

Mirrors python/triton_llm/ops/swiglu.py:54-76 of the reference (same signature, asserts and
output allocation) and calls the tcgen05 kernel ``tllm_swiglu``.
"""
from __future__ import annotations

import torch

from tritonllmcompiler_b200 import _lib


def swiglu(x: torch.Tensor, w1: torch.Tensor, w3: torch.Tensor) -> torch.Tensor:
    """x: [M,K], w1/w3: [K,N] -> [M,N] = silu(x @ w1) * (x @ w3).

    The tensor-core kernels need K and N multiples of 8 (and 16-byte-aligned rows); other
    shapes give the same results through a CUDA-core kernel at roughly 1/50 of the speed."""
    assert x.is_cuda and w1.is_cuda and w3.is_cuda
    assert x.dim() == 2 and w1.dim() == 2 and w3.dim() == 2
    m, k = x.shape
    k2, n = w1.shape
    assert k == k2 and w3.shape == (k, n)
    assert x.dtype in _lib.DTYPE_CODES and w1.dtype == x.dtype and w3.dtype == x.dtype
    out = torch.empty((m, n), device=x.device, dtype=x.dtype)
    if m == 0 or n == 0:
        return out
    x2 = x if x.stride(1) == 1 and x.stride(0) >= max(k, 1) else x.contiguous()
    a1 = w1 if w1.stride(1) == 1 and w1.stride(0) >= max(n, 1) else w1.contiguous()
    a3 = w3 if w3.stride(1) == 1 and w3.stride(0) >= max(n, 1) else w3.contiguous()
    lib = _lib.load()
    with _lib.on_device(x):
        _lib.check(
            lib.tllm_swiglu(
                x2.data_ptr(), a1.data_ptr(), a3.data_ptr(), out.data_ptr(), m, n, k,
                x2.stride(0), a1.stride(0), a3.stride(0), out.stride(0),
                _lib.DTYPE_CODES[x.dtype], _lib.stream_of(x),
            )
        )
    return out
