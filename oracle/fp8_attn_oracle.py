"""CPU oracle for FP8 (e4m3) flash attention -- TEST INFRASTRUCTURE ONLY.

The reference has no FP8 attention (python/triton_llm/ops/flash_attention.py:107-133 is
fp16/bf16); its FP8 counterpart is pinned to the reference's own definition applied to the
dequantized inputs: ``ops_oracle.flash_attention`` (python/triton_llm/reference/
flash_attention.py:12-29) of scale_q q8, scale_k k8 and scale_v v8 in fp32, unrounded.

The kernel rounds the probabilities P to e4m3 before P V (round to nearest even, 3 mantissa
bits: a relative error of at most 2^-4 for normal values, an absolute one of at most 2^-10
below 2^-6), while the row sums use P unrounded. So per output element
|kernel - oracle| <= 2^-4 * (softmax @ |v|) plus a small term for the subnormal P values and
the output rounding; ``error_bound`` returns the first term. Only ``tests/`` imports this.
"""
from __future__ import annotations

import numpy as np

from oracle.ops_oracle import flash_attention


def dequantize(t8, scale: float) -> np.ndarray:
    """e4m3 values (as float32) times their per-tensor scale, in fp32."""
    return np.asarray(t8, np.float32) * np.float32(scale)


def flash_attention_fp8(q8, k8, v8, scale_q: float, scale_k: float, scale_v: float, *,
                        causal: bool = False, sm_scale: float | None = None) -> np.ndarray:
    """q8, k8, v8: [B, H, S, D] float32 arrays holding e4m3 values (v8 NOT transposed)."""
    return flash_attention(dequantize(q8, scale_q), dequantize(k8, scale_k),
                           dequantize(v8, scale_v), causal=causal, sm_scale=sm_scale,
                           dtype="fp32")


def error_bound(q8, k8, v8, scale_q: float, scale_k: float, scale_v: float, *,
                causal: bool = False, sm_scale: float | None = None) -> np.ndarray:
    """2^-4 * (softmax @ |v|): the error that rounding P to e4m3 can cause (normal range)."""
    return np.float32(2.0 ** -4) * flash_attention(
        dequantize(q8, scale_q), dequantize(k8, scale_k), np.abs(dequantize(v8, scale_v)),
        causal=causal, sm_scale=sm_scale, dtype="fp32")
