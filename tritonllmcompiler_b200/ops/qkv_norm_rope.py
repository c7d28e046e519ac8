"""QKV projection with RMSNorm + RoPE fused into the GEMM epilogue.

The reference applies ``rmsnorm_rope`` (python/triton_llm/ops/rmsnorm_rope.py:51-75) to
projected q/k read back from HBM; this extension does it in the projection's epilogue.
Import from here; the package root keeps the reference's four exports.
"""
from __future__ import annotations

import torch

from tritonllmcompiler_b200 import _lib


def qkv_norm_rope(x: torch.Tensor, w: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor,
                  cos: torch.Tensor, sin: torch.Tensor, positions: torch.Tensor, *,
                  num_q_heads: int, num_kv_heads: int, eps: float = 1e-6) -> torch.Tensor:
    """x: [M, K]; w: [K, (Hq + 2*Hkv) * 128] (q | k | v heads); wq, wk: [128]; cos/sin:
    [P, 128]; positions: [M] int. Returns [M, (Hq + 2*Hkv) * 128]: q and k heads as
    ``rmsnorm_rope`` of the projection (cos/sin row = the token's position), v heads as
    projected."""
    assert x.is_cuda and x.dim() == 2 and w.dim() == 2 and x.shape[1] == w.shape[0]
    m, k = x.shape
    d = 128
    n = (num_q_heads + 2 * num_kv_heads) * d
    assert w.shape[1] == n
    assert x.dtype in _lib.DTYPE_CODES
    for t in (w, wq, wk, cos, sin):
        assert t.dtype == x.dtype
    assert wq.shape == (d,) and wk.shape == (d,) and cos.dim() == 2 and cos.shape[1] == d
    assert sin.shape == cos.shape and positions.shape == (m,)
    out = torch.empty((m, n), device=x.device, dtype=x.dtype)
    if m == 0 or n == 0:
        return out
    x, w = (t if t.stride(1) == 1 and t.stride(0) % 8 == 0 else t.contiguous() for t in (x, w))
    cos, sin = cos.contiguous(), sin.contiguous()
    pos = positions.to(torch.int32).contiguous()
    with _lib.on_device(x):
        _lib.check(_lib.load().tllm_qkv_norm_rope(
            x.data_ptr(), w.data_ptr(), wq.contiguous().data_ptr(), wk.contiguous().data_ptr(),
            cos.data_ptr(), sin.data_ptr(), cos.shape[0], cos.stride(0), sin.stride(0),
            pos.data_ptr(), out.data_ptr(), m, k, num_q_heads, num_kv_heads, d, x.stride(0),
            w.stride(0), out.stride(0), float(eps), _lib.DTYPE_CODES[x.dtype], _lib.stream_of(x)))
    return out
