"""CPU oracle for the FlashAttention backward pass -- TEST INFRASTRUCTURE ONLY.

The reference has the forward only; the function differentiated is its oracle
(python/triton_llm/reference/flash_attention.py:12-29): S = q k^T * scale, top-left causal
mask (triu(1) -> -inf), P = softmax(S), O = P v. Its gradients, in fp32:
dV = P^T dO, dP = dO V^T, dS = P * (dP - rowsum(dP * P)), dQ = scale * dS K,
dK = scale * dS^T Q. ``lse`` is the forward's per-row log2 normaliser in units of
s * scale * log2(e). Only ``tests/`` imports this module.
"""
from __future__ import annotations

import numpy as np

from oracle.ops_oracle import round_to

LOG2E = 1.4426950408889634


def forward_lse(q, k, causal: bool, sm_scale: float) -> np.ndarray:
    """[B, H, Sq] log2 normalisers (rows with no visible key give -inf)."""
    s = np.matmul(np.asarray(q, np.float32), np.swapaxes(np.asarray(k, np.float32), -1, -2))
    s = s * np.float32(sm_scale * LOG2E)
    if causal:
        m, n = s.shape[-2:]
        s = np.where(np.triu(np.ones((m, n), bool), k=1), np.float32(-np.inf), s)
    mx = np.max(s, axis=-1, keepdims=True)
    with np.errstate(divide="ignore", invalid="ignore"):
        return (mx + np.log2(np.sum(np.exp2(s - mx), axis=-1, keepdims=True)))[..., 0]


def flash_attention_backward(q, k, v, dout, *, causal: bool = False, sm_scale: float | None = None,
                             dtype: str = "fp16"):
    """(dq, dk, dv) of the reference's flash_attention at (q, k, v) for output gradient dout,
    each rounded to the I/O dtype. q: [B,H,Sq,D], k/v: [B,H,Sk,D], dout: [B,H,Sq,D]."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    do = np.asarray(dout, np.float32)
    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    s = np.matmul(q, np.swapaxes(k, -1, -2)) * np.float32(sm_scale)
    if causal:
        m, n = s.shape[-2:]
        s = np.where(np.triu(np.ones((m, n), bool), k=1), np.float32(-np.inf), s)
    mx = np.max(s, axis=-1, keepdims=True)
    e = np.exp(s - mx)
    p = e / np.sum(e, axis=-1, keepdims=True)
    dv = np.matmul(np.swapaxes(p, -1, -2), do)
    dp = np.matmul(do, np.swapaxes(v, -1, -2))
    ds = p * (dp - np.sum(dp * p, axis=-1, keepdims=True))
    dq = np.matmul(ds, k) * np.float32(sm_scale)
    dk = np.matmul(np.swapaxes(ds, -1, -2), q) * np.float32(sm_scale)
    return round_to(dq, dtype), round_to(dk, dtype), round_to(dv, dtype)
