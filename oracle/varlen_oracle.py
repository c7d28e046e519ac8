"""CPU oracle for variable-length (packed) flash attention -- TEST INFRASTRUCTURE ONLY.

The reference's flash_attention takes padded [B, H, S, D] tensors
(python/triton_llm/ops/flash_attention.py:107-133). Its packed counterpart is pinned here
to the same per-sequence definition: sequence b's queries are rows [cu_q[b], cu_q[b+1]) of
q [total_q, H, D], its keys rows [cu_k[b], cu_k[b+1]) of k/v [total_k, Hkv, D], and each
(sequence, query head h) is ``ops_oracle.flash_attention``
(python/triton_llm/reference/flash_attention.py:12-29) against key/value head
h // (H / Hkv), with its top-left causal mask. Only ``tests/`` imports this module.
"""
from __future__ import annotations

import numpy as np

from oracle.ops_oracle import flash_attention


def flash_attention_varlen(q, k, v, cu_q, cu_k, *, causal: bool = False,
                           sm_scale: float | None = None, dtype: str = "fp16") -> np.ndarray:
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    H, Hkv = q.shape[1], k.shape[1]
    G = H // Hkv
    out = np.zeros_like(q)
    for b in range(len(cu_q) - 1):
        q0, q1 = int(cu_q[b]), int(cu_q[b + 1])
        k0, k1 = int(cu_k[b]), int(cu_k[b + 1])
        if q1 == q0:
            continue
        qs = np.transpose(q[q0:q1], (1, 0, 2))[None]                   # [1, H, Sq, D]
        ks = np.repeat(np.transpose(k[k0:k1], (1, 0, 2)), G, axis=0)[None]  # [1, H, Sk, D]
        vs = np.repeat(np.transpose(v[k0:k1], (1, 0, 2)), G, axis=0)[None]
        if k1 == k0:
            out[q0:q1] = np.nan
            continue
        o = flash_attention(qs, ks, vs, causal=causal, sm_scale=sm_scale, dtype=dtype)
        out[q0:q1] = np.transpose(o[0], (1, 0, 2))
    return out
