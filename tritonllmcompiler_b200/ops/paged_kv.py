"""Operators either side of paged decode: filling the paged KV cache.

The reference decodes from a paged cache (python/triton_llm/ops/paged_attention.py:92-128)
but has no operator that writes it; these use its layout (token t of sequence b at
cache[block_tables[b, t // block_size], t % block_size, h, :],
python/triton_llm/reference/paged_attention.py:29-37). They are extensions: the package
root and ``ops`` keep the reference's four exports, and these are imported from this module.

Unlike the four reference operators, which allocate their outputs, these update the caches
in place (the cache is the state being built).
"""
from __future__ import annotations

import torch

from tritonllmcompiler_b200 import _lib


def _vec_ok(t: torch.Tensor) -> bool:
    s = t.stride()
    return s[-1] == 1 and all(x % 8 == 0 for x in s[:-1]) and t.data_ptr() % 16 == 0


def _check_common(k_new, v_new, k_cache, v_cache, block_tables, start_pos, n_new, block_size):
    assert k_new.is_cuda and k_new.dim() == 4 and v_new.shape == k_new.shape
    b, t, h, d = k_new.shape
    assert d in (16, 32, 64, 128)
    assert block_size >= 1
    assert k_new.dtype in _lib.DTYPE_CODES
    assert v_new.dtype == k_new.dtype and k_cache.dtype == k_new.dtype and v_cache.dtype == k_new.dtype
    assert k_cache.dim() == 4 and tuple(k_cache.shape[1:]) == (block_size, h, d)
    assert tuple(v_cache.shape) == tuple(k_cache.shape)
    assert _vec_ok(k_cache) and _vec_ok(v_cache), "caches need unit inner stride and 16-byte rows"
    assert block_tables.dim() == 2 and block_tables.shape[0] == b
    assert start_pos.shape == (b,)
    assert n_new is None or n_new.shape == (b,)
    bt = block_tables if block_tables.dtype == torch.int32 else block_tables.to(torch.int32)
    sp = start_pos.to(torch.int32).contiguous()
    nn = None if n_new is None else n_new.to(torch.int32).contiguous()
    kn = k_new if _vec_ok(k_new) else k_new.contiguous()
    vn = v_new if _vec_ok(v_new) else v_new.contiguous()
    return b, t, h, d, bt, sp, nn, kn, vn


def paged_kv_append(k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor,
                    v_cache: torch.Tensor, block_tables: torch.Tensor, start_pos: torch.Tensor,
                    n_new: torch.Tensor | None = None, *, block_size: int) -> None:
    """Writes token t of k_new[b]/v_new[b] ([B, T, H, D]) at position start_pos[b] + t of
    sequence b, for t < n_new[b] (all T when n_new is None). Caches: [num_blocks,
    block_size, H, D], updated in place. Positions past the block table or table entries
    outside the pool are skipped and flagged (``_lib.debug_status()`` returns 0x200)."""
    b, t, h, d, bt, sp, nn, kn, vn = _check_common(k_new, v_new, k_cache, v_cache, block_tables,
                                                   start_pos, n_new, block_size)
    if b * t * h == 0:
        return
    lib = _lib.load()
    with _lib.on_device(k_new):
        _lib.check(lib.tllm_paged_kv_append(
            kn.data_ptr(), vn.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), bt.data_ptr(),
            sp.data_ptr(), None if nn is None else nn.data_ptr(), b, t, h, d, block_size,
            bt.shape[1], k_cache.shape[0], _lib.strides(kn), _lib.strides(vn),
            _lib.strides(k_cache), _lib.strides(v_cache), _lib.strides(bt),
            _lib.DTYPE_CODES[k_new.dtype], _lib.stream_of(k_new)))


def paged_kv_append_rope(k_new: torch.Tensor, v_new: torch.Tensor, weight: torch.Tensor,
                         cos: torch.Tensor, sin: torch.Tensor, k_cache: torch.Tensor,
                         v_cache: torch.Tensor, block_tables: torch.Tensor,
                         start_pos: torch.Tensor, n_new: torch.Tensor | None = None, *,
                         block_size: int, eps: float = 1e-6) -> None:
    """``paged_kv_append`` with K passed through ``rmsnorm_rope`` first, fused: the cache
    receives exactly what ``rmsnorm_rope`` returns for each new K row, with the cos/sin row
    ([P, D] tables) of the token's absolute position start_pos[b] + t."""
    b, t, h, d, bt, sp, nn, kn, vn = _check_common(k_new, v_new, k_cache, v_cache, block_tables,
                                                   start_pos, n_new, block_size)
    assert weight.shape == (d,) and cos.dim() == 2 and cos.shape[1] == d and sin.shape == cos.shape
    assert weight.dtype == k_new.dtype and cos.dtype == k_new.dtype and sin.dtype == k_new.dtype
    if b * t * h == 0:
        return
    w = weight.contiguous()
    cs = cos if _vec_ok(cos) else cos.contiguous()
    sn = sin if _vec_ok(sin) else sin.contiguous()
    lib = _lib.load()
    with _lib.on_device(k_new):
        _lib.check(lib.tllm_paged_kv_append_rope(
            kn.data_ptr(), vn.data_ptr(), w.data_ptr(), cs.data_ptr(), sn.data_ptr(),
            cs.shape[0], cs.stride(0), sn.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
            bt.data_ptr(), sp.data_ptr(), None if nn is None else nn.data_ptr(), b, t, h, d,
            block_size, bt.shape[1], k_cache.shape[0], _lib.strides(kn), _lib.strides(vn),
            _lib.strides(k_cache), _lib.strides(v_cache), _lib.strides(bt), float(eps),
            _lib.DTYPE_CODES[k_new.dtype], _lib.stream_of(k_new)))


def paged_attention_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                            block_tables: torch.Tensor, context_lens: torch.Tensor, *,
                            block_size: int, sm_scale: float | None = None,
                            causal: bool = True) -> torch.Tensor:
    """Attention of Sq >= 1 new query tokens per sequence over the paged cache.

    q: [B, Hq, Sq, D]; caches: [num_blocks, block_size, Hkv, D] with Hq % Hkv == 0 (grouped
    query heads); context_lens[b] counts the new tokens, which are already in the cache.
    Query s sits at position context_lens[b] - Sq + s; with causal it sees keys up to its own
    position. Returns a new [B, Hq, Sq, D] tensor. With Sq = 1 and Hq = Hkv it computes what
    ``paged_attention`` computes.
    """
    assert q.is_cuda and q.dim() == 4
    b, hq, sq, d = q.shape
    assert d in (16, 32, 64, 128)
    assert block_size in (16, 32, 64)
    assert q.dtype in _lib.DTYPE_CODES and k_cache.dtype == q.dtype and v_cache.dtype == q.dtype
    assert k_cache.dim() == 4 and k_cache.shape[1] == block_size and k_cache.shape[3] == d
    hkv = k_cache.shape[2]
    assert hkv >= 1 and hq % hkv == 0
    assert tuple(v_cache.shape) == tuple(k_cache.shape)
    assert block_tables.dim() == 2 and block_tables.shape[0] == b and context_lens.shape == (b,)
    if sm_scale is None:
        sm_scale = d ** -0.5
    out = torch.empty((b, hq, sq, d), device=q.device, dtype=q.dtype)
    if b == 0 or hq == 0 or sq == 0:
        return out
    qq = q if _vec_ok(q) else q.contiguous()
    kc = k_cache if _vec_ok(k_cache) else k_cache.contiguous()
    vc = v_cache if _vec_ok(v_cache) else v_cache.contiguous()
    bt = block_tables if block_tables.dtype == torch.int32 else block_tables.to(torch.int32)
    cl = context_lens.to(torch.int32).contiguous()
    lib = _lib.load()
    with _lib.on_device(q):
        ws_bytes = lib.tllm_paged_prefill_workspace_size(b, hq, hkv, sq, d, block_size,
                                                         bt.shape[1])
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
        _lib.check(lib.tllm_paged_prefill(
            qq.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), cl.data_ptr(),
            out.data_ptr(), ws.data_ptr(), ws_bytes, b, hq, hkv, sq, d, block_size, bt.shape[1],
            kc.shape[0], _lib.strides(qq), _lib.strides(kc), _lib.strides(vc), _lib.strides(bt),
            _lib.strides(out), float(sm_scale), int(bool(causal)), _lib.DTYPE_CODES[q.dtype],
            _lib.stream_of(q)))
    return out
