"""FP8 (e4m3) SwiGLU on B200: the tcgen05 kind::f8f6f4 path.

An extension of the reference's fp16 ``swiglu`` (python/triton_llm/ops/swiglu.py:54-76) to
8-bit inputs with per-tensor scales: out = silu(sx*s1 * x@w1) * (sx*s3 * x@w3). The weights
are passed transposed ([N, K], K contiguous), the layout FP8 weights are stored in.
"""
from __future__ import annotations

import torch

from tritonllmcompiler_b200 import _lib

E4M3_MAX = 448.0


def quantize_e4m3(t: torch.Tensor):
    """(t8, scale): per-tensor e4m3 quantization with t ~= t8.float() * scale."""
    amax = t.abs().amax().float().clamp(min=1e-12)
    scale = (amax / E4M3_MAX).item()
    return (t.float() / scale).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn), scale


def swiglu_fp8(x8: torch.Tensor, w1t8: torch.Tensor, w3t8: torch.Tensor, scale_x: float,
               scale_w1: float, scale_w3: float, out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """x8: [M, K], w1t8/w3t8: [N, K], all torch.float8_e4m3fn; returns [M, N] in out_dtype."""
    assert x8.is_cuda and x8.dim() == 2 and w1t8.dim() == 2 and w3t8.shape == w1t8.shape
    assert x8.dtype == torch.float8_e4m3fn and w1t8.dtype == x8.dtype and w3t8.dtype == x8.dtype
    assert out_dtype in _lib.DTYPE_CODES
    m, k = x8.shape
    n, k2 = w1t8.shape
    assert k == k2
    out = torch.empty((m, n), device=x8.device, dtype=out_dtype)
    if m == 0 or n == 0:
        return out
    x8, w1t8, w3t8 = (t if t.stride(1) == 1 else t.contiguous() for t in (x8, w1t8, w3t8))
    with _lib.on_device(x8):
        _lib.check(_lib.load().tllm_swiglu_fp8(
            x8.data_ptr(), w1t8.data_ptr(), w3t8.data_ptr(), out.data_ptr(), m, n, k, x8.stride(0),
            w1t8.stride(0), w3t8.stride(0), out.stride(0), float(scale_x), float(scale_w1),
            float(scale_w3), _lib.DTYPE_CODES[out_dtype], _lib.stream_of(x8)))
    return out
