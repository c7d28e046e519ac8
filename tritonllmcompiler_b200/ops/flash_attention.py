"""FlashAttention forward on B200: drop-in for ``triton_llm.ops.flash_attention``.

Mirrors python/triton_llm/ops/flash_attention.py:107-133 of the reference (same signature,
same defaults, same AssertionError/ValueError checks, fresh contiguous output) and calls the
tcgen05/TMEM kernel ``tllm_flash_attn_fwd`` of libtllm_sm100a.so.
"""
from __future__ import annotations

import torch

from tritonllmcompiler_b200 import _lib


def _tma_ready(t: torch.Tensor) -> bool:
    s = t.stride()
    return s[3] == 1 and all(x % 8 == 0 for x in s[:3]) and t.data_ptr() % 16 == 0


def flash_attention(q, k, v, *, causal: bool = False, sm_scale: float | None = None):
    """q/k/v: [B, H, S, D] fp16 or bf16. Online softmax, no SxS score matrix in HBM.

    Returns a new contiguous [B, H, Sq, D] tensor of q.dtype. The causal mask is top-left
    aligned (query i sees keys j <= i), as in the reference.
    """
    assert q.is_cuda and k.is_cuda and v.is_cuda
    if q.dtype == torch.bfloat16:
        major, _ = torch.cuda.get_device_capability(q.device)
        if major < 8:
            raise ValueError("BF16 flash_attention requires sm_80+; use FP16 on V100")
    b, h, seqlen_q, d = q.shape
    seqlen_k = k.shape[2]
    assert d in (16, 32, 64, 128)
    assert q.dtype in _lib.DTYPE_CODES and k.dtype == q.dtype and v.dtype == q.dtype
    assert tuple(k.shape) == (b, h, seqlen_k, d) and tuple(v.shape) == (b, h, seqlen_k, d)
    if sm_scale is None:
        sm_scale = d ** -0.5
    q2 = q if _tma_ready(q) else q.contiguous()
    k2 = k if _tma_ready(k) else k.contiguous()
    v2 = v if _tma_ready(v) else v.contiguous()
    out = torch.empty((b, h, seqlen_q, d), device=q.device, dtype=q.dtype)
    lib = _lib.load()
    with _lib.on_device(q):
        _lib.check(
            lib.tllm_flash_attn_fwd(
                q2.data_ptr(), k2.data_ptr(), v2.data_ptr(), out.data_ptr(),
                b, h, seqlen_q, seqlen_k, d,
                _lib.strides(q2), _lib.strides(k2), _lib.strides(v2), _lib.strides(out),
                float(sm_scale), int(bool(causal)), _lib.DTYPE_CODES[q.dtype],
                _lib.stream_of(q),
            )
        )
    return out
