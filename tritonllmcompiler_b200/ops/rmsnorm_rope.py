"""Fused RMSNorm + RoPE on B200: drop-in for ``triton_llm.ops.rmsnorm_rope``.

Mirrors python/triton_llm/ops/rmsnorm_rope.py:51-75 of the reference (same signature, asserts
and ``empty_like`` output) and calls ``tllm_rmsnorm_rope``. The normalised value is rounded
to the I/O dtype before RoPE, as the reference's oracle does
(python/triton_llm/reference/norm_rope.py:15).
"""
from __future__ import annotations

import torch

from tritonllmcompiler_b200 import _lib


def rmsnorm_rope(
    x: torch.Tensor,
    weight: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    eps: float = 1e-6,
) -> torch.Tensor:
    """x: [B,S,H,D]; weight: [D]; cos/sin: [S,D]. Single fused kernel."""
    assert x.is_cuda and x.dim() == 4
    b, s, h, d = x.shape
    assert d % 2 == 0 and d in (16, 32, 64, 128)
    assert weight.shape == (d,)
    assert cos.shape == (s, d) and sin.shape == (s, d)
    assert x.dtype in _lib.DTYPE_CODES
    # The kernel reads weight/cos/sin in the I/O dtype.
    w = weight if weight.dtype == x.dtype else weight.to(x.dtype)
    c = cos if cos.dtype == x.dtype else cos.to(x.dtype)
    sn = sin if sin.dtype == x.dtype else sin.to(x.dtype)
    out = torch.empty_like(x)
    if out.numel() == 0:
        return out
    lib = _lib.load()
    with _lib.on_device(x):
        _lib.check(
            lib.tllm_rmsnorm_rope(
                x.data_ptr(), w.data_ptr(), c.data_ptr(), sn.data_ptr(), out.data_ptr(),
                b, s, h, d, _lib.strides(x), w.stride(0), _lib.strides(c), _lib.strides(sn),
                _lib.strides(out), float(eps), _lib.DTYPE_CODES[x.dtype], _lib.stream_of(x),
            )
        )
    return out
