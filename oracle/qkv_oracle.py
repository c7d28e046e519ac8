"""CPU oracle for the fused QKV projection + RMSNorm + RoPE -- TEST INFRASTRUCTURE ONLY.

Composes pinned definitions: the projection x @ w in fp32 rounded to the I/O dtype (what a
separate GEMM stores), then, per q and k head, ``ops_oracle.rmsnorm_rope``
(python/triton_llm/reference/norm_rope.py:12-40) with the cos/sin row of each token's
position; v heads are the rounded projection. Only ``tests/`` imports this module.
"""
from __future__ import annotations

import numpy as np

from oracle.ops_oracle import rmsnorm_rope, round_to


def qkv_norm_rope(x, w, wq, wk, cos, sin, positions, *, num_q_heads: int, num_kv_heads: int,
                  eps: float = 1e-6, dtype: str = "fp16") -> np.ndarray:
    proj = round_to(np.asarray(x, np.float32) @ np.asarray(w, np.float32), dtype)
    m = proj.shape[0]
    d = 128
    heads = proj.reshape(m, num_q_heads + 2 * num_kv_heads, d)
    pos = np.clip(np.asarray(positions), 0, np.asarray(cos).shape[0] - 1)
    c = np.asarray(cos, np.float32)[pos]  # [M, D]
    s = np.asarray(sin, np.float32)[pos]
    out = heads.copy()
    for lo, hi, wt in [(0, num_q_heads, wq), (num_q_heads, num_q_heads + num_kv_heads, wk)]:
        if hi > lo:
            # rmsnorm_rope takes [B, S, H, D] with cos/sin [S, D]: one "sequence" of M tokens
            out[:, lo:hi] = rmsnorm_rope(heads[None, :, lo:hi], wt, c, s, eps, dtype=dtype)[0]
    return out.reshape(m, -1)
