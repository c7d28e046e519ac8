"""Paged-KV decode attention on B200: drop-in for ``triton_llm.ops.paged_attention``.

Mirrors python/triton_llm/ops/paged_attention.py:92-128 of the reference (same signature and
asserts, output [B, H, 1, D]) and calls the split-KV kernel ``tllm_paged_attn_decode``.
Unlike the reference, no host synchronisation happens: the reference reads
``context_lens.max().item()`` to size its loop (:113); here context lengths are read on the
device and the launch is sized from ``block_tables.shape[1]``.
"""
from __future__ import annotations

import torch

from tritonllmcompiler_b200 import _lib


def paged_attention(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    *,
    block_size: int,
    sm_scale: float | None = None,
) -> torch.Tensor:
    """q: [B,H,1,D]; caches: [num_blocks, block_size, H, D]; block_tables: [B, max_blocks]."""
    assert q.is_cuda
    b, h, m, d = q.shape
    assert m == 1, "paged_attention decode kernel expects seqlen_q == 1"
    assert d in (16, 32, 64, 128)
    assert block_size in (16, 32, 64)
    assert q.dtype in _lib.DTYPE_CODES and k_cache.dtype == q.dtype and v_cache.dtype == q.dtype
    assert k_cache.dim() == 4 and tuple(k_cache.shape[1:]) == (block_size, h, d)
    assert tuple(v_cache.shape) == tuple(k_cache.shape)
    assert block_tables.dim() == 2 and block_tables.shape[0] == b and context_lens.shape == (b,)
    if sm_scale is None:
        sm_scale = d ** -0.5

    out = torch.empty((b, h, 1, d), device=q.device, dtype=q.dtype)
    if b == 0 or h == 0:
        return out
    max_blocks = block_tables.shape[1]
    num_blocks = k_cache.shape[0]
    bt = block_tables if block_tables.dtype == torch.int32 else block_tables.to(torch.int32)
    cl = context_lens.to(torch.int32).contiguous()

    def cache_ok(c):
        s = c.stride()
        return s[3] == 1 and all(x % 8 == 0 for x in s[:3]) and c.data_ptr() % 16 == 0

    kc = k_cache if cache_ok(k_cache) else k_cache.contiguous()
    vc = v_cache if cache_ok(v_cache) else v_cache.contiguous()
    lib = _lib.load()
    with _lib.on_device(q):
        ws_bytes = lib.tllm_paged_attn_workspace_size(b, h, d, block_size, max_blocks)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
        _lib.check(
            lib.tllm_paged_attn_decode(
                q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), cl.data_ptr(),
                out.data_ptr(), ws.data_ptr(), ws_bytes,
                b, h, d, block_size, max_blocks, num_blocks,
                _lib.strides(q), _lib.strides(kc), _lib.strides(vc), _lib.strides(bt),
                _lib.strides(out), float(sm_scale), _lib.DTYPE_CODES[q.dtype],
                _lib.stream_of(q),
            )
        )
    return out
