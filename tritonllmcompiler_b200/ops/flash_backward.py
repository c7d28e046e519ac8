"""FlashAttention backward on B200, and a differentiable attention built on it.

The reference's ``flash_attention`` (python/triton_llm/ops/flash_attention.py:107-133) is
forward only. ``flash_attention_fwd_lse`` runs the same forward and also returns each row's
log2 softmax normaliser; ``flash_attention_backward`` turns (q, k, v, o, lse, dout) into
(dq, dk, dv); ``flash_attention_train`` wraps both in a ``torch.autograd.Function``. These are
extensions: the package root and ``ops`` keep the reference's four exports.
"""
from __future__ import annotations

import torch

from tritonllmcompiler_b200 import _lib


def _ok(t: torch.Tensor) -> bool:
    s = t.stride()
    return s[3] == 1 and all(x % 8 == 0 for x in s[:3]) and t.data_ptr() % 16 == 0


def flash_attention_fwd_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                            causal: bool = False, sm_scale: float | None = None):
    """(o, lse): ``flash_attention``'s output and the fp32 [B, H, Sq] log2 normalisers."""
    assert q.is_cuda and q.dim() == 4 and k.shape == v.shape and k.shape[:2] == q.shape[:2]
    b, h, sq, d = q.shape
    sk = k.shape[2]
    assert d in (16, 32, 64, 128) and k.shape[3] == d
    assert q.dtype in _lib.DTYPE_CODES and k.dtype == q.dtype and v.dtype == q.dtype
    if sm_scale is None:
        sm_scale = d ** -0.5
    q, k, v = (t if _ok(t) else t.contiguous() for t in (q, k, v))
    o = torch.empty((b, h, sq, d), device=q.device, dtype=q.dtype)
    lse = torch.empty((b, h, sq), device=q.device, dtype=torch.float32)
    if b * h * sq == 0:
        return o, lse
    with _lib.on_device(q):
        _lib.check(_lib.load().tllm_flash_attn_fwd_lse(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), b, h, sq, sk, d,
            _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(o), float(sm_scale),
            int(bool(causal)), _lib.DTYPE_CODES[q.dtype], _lib.stream_of(q)))
    return o, lse


def flash_attention_backward(q, k, v, o, lse, dout, *, causal: bool = False,
                             sm_scale: float | None = None):
    """(dq, dk, dv) for ``flash_attention`` at (q, k, v) given its output o, the lse from
    ``flash_attention_fwd_lse`` and the output gradient dout. Head dims 64 and 128."""
    assert q.is_cuda and q.dim() == 4 and k.shape == v.shape and k.shape[:2] == q.shape[:2]
    b, h, sq, d = q.shape
    sk = k.shape[2]
    assert d in (64, 128) and k.shape[3] == d
    assert o.shape == q.shape and dout.shape == q.shape and lse.shape == (b, h, sq)
    assert lse.dtype == torch.float32
    for t in (k, v, o, dout):
        assert t.dtype == q.dtype
    if sm_scale is None:
        sm_scale = d ** -0.5
    q, k, v, o, dout = (t if _ok(t) else t.contiguous() for t in (q, k, v, o, dout))
    lse = lse.contiguous()
    dq = torch.empty_like(q, memory_format=torch.contiguous_format)
    dk = torch.empty_like(k, memory_format=torch.contiguous_format)
    dv = torch.empty_like(v, memory_format=torch.contiguous_format)
    if b * h == 0 or (sq == 0 and sk == 0):
        return dq, dk, dv
    lib = _lib.load()
    with _lib.on_device(q):
        ws_bytes = lib.tllm_flash_attn_bwd_workspace_size(b, h, sq, d)
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=q.device)
        _lib.check(lib.tllm_flash_attn_bwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr(),
            lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ws.data_ptr(), ws_bytes,
            b, h, sq, sk, d, _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(o),
            _lib.strides(dout), _lib.strides(dq), _lib.strides(dk), _lib.strides(dv),
            float(sm_scale), int(bool(causal)), _lib.DTYPE_CODES[q.dtype], _lib.stream_of(q)))
    return dq, dk, dv


class _FlashAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, sm_scale):
        o, lse = flash_attention_fwd_lse(q, k, v, causal=causal, sm_scale=sm_scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal, ctx.sm_scale = causal, sm_scale
        return o

    @staticmethod
    def backward(ctx, dout):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = flash_attention_backward(q, k, v, o, lse, dout, causal=ctx.causal,
                                              sm_scale=ctx.sm_scale)
        return dq, dk, dv, None, None


def flash_attention_train(q, k, v, *, causal: bool = False, sm_scale: float | None = None):
    """``flash_attention`` with a backward pass (torch autograd)."""
    return _FlashAttention.apply(q, k, v, causal, sm_scale)
