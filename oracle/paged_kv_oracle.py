"""CPU oracle for the paged-KV operators around decode -- TEST INFRASTRUCTURE ONLY.

The reference (xdlhzdh/TritonLLMCompiler) has the decode step only: `paged_attention` with one
query token and equal query/KV head counts (python/triton_llm/ops/paged_attention.py:105).
The steps either side of it are built here on the reference's own cache layout and numerics:

* the cache layout and addressing of python/triton_llm/reference/paged_attention.py:29-37:
  token t of sequence b lives at cache[block_tables[b, t // block_size], t % block_size, h];
* RMSNorm + RoPE exactly as python/triton_llm/reference/norm_rope.py:12-40 (``rmsnorm_rope``
  of ``ops_oracle``), with the cos/sin row taken at each token's absolute position;
* attention exactly as python/triton_llm/reference/flash_attention.py:12-29 (fp32 scores,
  softmax, fp32 probs @ v, one rounding), with a causal mask aligned to the END of the
  context (query s of Sq new tokens sits at position context_len - Sq + s) and grouped
  query heads (query head hq reads KV head hq // (Hq / Hkv)).

With Sq = 1 and Hq = Hkv, ``paged_attention_prefill`` is the reference's
``paged_attention_ref`` (the test suite checks that). Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs import this module.
"""
from __future__ import annotations

import numpy as np

from oracle.ops_oracle import rmsnorm_rope, round_to


def _slots(block_tables, start_pos, n_new, t_max: int, block_size: int):
    """(b, t, physical block, offset) for every appended token, in (b, t) order."""
    out = []
    for b in range(len(start_pos)):
        n = t_max if n_new is None else int(n_new[b])
        for t in range(min(n, t_max)):
            pos = int(start_pos[b]) + t
            out.append((b, t, int(block_tables[b, pos // block_size]), pos % block_size))
    return out


def paged_kv_append(k_new, v_new, k_cache, v_cache, block_tables, start_pos, n_new=None, *,
                    block_size: int):
    """Copies of the caches with token t of k_new[b]/v_new[b] written at position
    start_pos[b] + t of sequence b (t < n_new[b], all T tokens when n_new is None).

    k_new/v_new: [B, T, Hkv, D]; caches: [num_blocks, block_size, Hkv, D].
    """
    kc = np.array(k_cache, dtype=np.float32, copy=True)
    vc = np.array(v_cache, dtype=np.float32, copy=True)
    k_new = np.asarray(k_new, np.float32)
    v_new = np.asarray(v_new, np.float32)
    for b, t, phys, off in _slots(np.asarray(block_tables), start_pos, n_new, k_new.shape[1],
                                  block_size):
        kc[phys, off] = k_new[b, t]
        vc[phys, off] = v_new[b, t]
    return kc, vc


def paged_kv_append_rope(k_new, v_new, weight, cos, sin, k_cache, v_cache, block_tables,
                         start_pos, n_new=None, *, block_size: int, eps: float = 1e-6,
                         dtype: str = "fp16"):
    """As ``paged_kv_append``, with K passed through RMSNorm + RoPE first; the RoPE row of
    token t of sequence b is cos/sin[start_pos[b] + t] (cos/sin: [P, D])."""
    k_new = np.asarray(k_new, np.float32)
    B, T = k_new.shape[:2]
    cos = np.asarray(cos, np.float32)
    sin = np.asarray(sin, np.float32)
    k_rot = np.empty_like(k_new)
    for b in range(B):
        pos = int(start_pos[b]) + np.arange(T)
        pos = np.minimum(pos, cos.shape[0] - 1)  # rows past the table are never written
        k_rot[b:b + 1] = rmsnorm_rope(k_new[b:b + 1], weight, cos[pos], sin[pos], eps,
                                      dtype=dtype)
    return paged_kv_append(k_rot, v_new, k_cache, v_cache, block_tables, start_pos, n_new,
                           block_size=block_size)


def paged_attention_prefill(q, k_cache, v_cache, block_tables, context_lens, *,
                            block_size: int, sm_scale: float | None = None,
                            causal: bool = True, dtype: str = "fp16") -> np.ndarray:
    """Attention of Sq new query tokens per sequence over its paged context.

    q: [B, Hq, Sq, D]; caches: [num_blocks, block_size, Hkv, D] with Hq % Hkv == 0;
    context_lens[b] counts the new tokens too. Query s sees key t when t < context_len and,
    with causal, t <= context_len - Sq + s. A query that sees no key gives NaN (0/0), as the
    reference does for an empty context.
    """
    q = np.asarray(q, np.float32)
    B, Hq, Sq, D = q.shape
    Hkv = k_cache.shape[2]
    G = Hq // Hkv
    if sm_scale is None:
        sm_scale = D ** -0.5
    block_tables = np.asarray(block_tables)
    out = np.empty_like(q)
    for b in range(B):
        clen = int(context_lens[b])
        nblocks = (clen + block_size - 1) // block_size
        phys = block_tables[b, :nblocks].astype(np.int64)
        k = np.asarray(k_cache[phys], np.float32).reshape(-1, Hkv, D)[:clen]
        v = np.asarray(v_cache[phys], np.float32).reshape(-1, Hkv, D)[:clen]
        visible = np.ones((Sq, clen), dtype=bool)
        if causal:
            pos = clen - Sq + np.arange(Sq)
            visible = np.arange(clen)[None, :] <= pos[:, None]
        for hq in range(Hq):
            kvh = hq // G
            s = (q[b, hq] @ k[:, kvh].T) * np.float32(sm_scale)
            s = np.where(visible, s, np.float32(-np.inf))
            with np.errstate(invalid="ignore", divide="ignore"):
                m = np.max(s, axis=-1, keepdims=True) if clen else np.zeros((Sq, 1), np.float32)
                e = np.exp(s - m)
                p = e / np.sum(e, axis=-1, keepdims=True)
            out[b, hq] = p @ v[:, kvh] if clen else np.float32(np.nan)
    return round_to(out, dtype)
