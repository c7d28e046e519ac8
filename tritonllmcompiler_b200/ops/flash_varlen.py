"""Variable-length (packed) flash attention forward on B200.

The reference's ``flash_attention`` (python/triton_llm/ops/flash_attention.py:107-133) takes
padded [B, H, S, D] batches; prefill of sequences of different lengths wastes the padding.
This packed form is an extension with the same per-sequence result: the sequences are
concatenated along the row axis and delimited by cumulative lengths, as in FlashAttention's
varlen interface, and key/value heads may be shared by groups of query heads. The package
root and ``ops`` keep the reference's four exports; import this from here.
"""
from __future__ import annotations

import torch

from tritonllmcompiler_b200 import _lib


def flash_attention_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor,
                           max_seqlen_q: int, max_seqlen_k: int, *, causal: bool = False,
                           sm_scale: float | None = None) -> torch.Tensor:
    """q: [total_q, H, D]; k, v: [total_k, Hkv, D] with H % Hkv == 0; cu_seqlens_q/k: [B + 1]
    int32 cumulative lengths (on the device); max_seqlen_q/k bound every sequence's lengths.
    Returns a new [total_q, H, D] tensor; sequence b's rows are computed as
    ``flash_attention`` of its own rows (top-left causal mask), query head h reading key/value
    head h // (H // Hkv)."""
    assert q.is_cuda and q.dim() == 3 and k.dim() == 3 and v.shape == k.shape
    total_q, h, d = q.shape
    total_k, hkv, d2 = k.shape
    assert d == d2 and d in (16, 32, 64, 128)
    assert hkv >= 1 and h % hkv == 0
    assert q.dtype in _lib.DTYPE_CODES and k.dtype == q.dtype and v.dtype == q.dtype
    assert cu_seqlens_q.dim() == 1 and cu_seqlens_k.shape == cu_seqlens_q.shape
    b = cu_seqlens_q.shape[0] - 1
    assert b >= 0
    if sm_scale is None:
        sm_scale = d ** -0.5
    out = torch.empty_like(q, memory_format=torch.contiguous_format)
    if b == 0 or total_q == 0 or max_seqlen_q == 0:
        return out

    def ok(t):
        s = t.stride()
        return s[2] == 1 and s[0] % 8 == 0 and s[1] % 8 == 0 and t.data_ptr() % 16 == 0

    qq = q if ok(q) else q.contiguous()
    kk = k if ok(k) else k.contiguous()
    vv = v if ok(v) else v.contiguous()
    cq = cu_seqlens_q.to(torch.int32).contiguous()
    ck = cu_seqlens_k.to(torch.int32).contiguous()
    lib = _lib.load()
    with _lib.on_device(q):
        _lib.check(lib.tllm_flash_attn_varlen_fwd(
            qq.data_ptr(), kk.data_ptr(), vv.data_ptr(), out.data_ptr(), cq.data_ptr(),
            ck.data_ptr(), b, h, hkv, total_q, total_k, int(max_seqlen_q), int(max_seqlen_k), d,
            _lib.strides(qq), _lib.strides(kk), _lib.strides(vv), _lib.strides(out),
            float(sm_scale), int(bool(causal)), _lib.DTYPE_CODES[q.dtype], _lib.stream_of(q)))
    return out
