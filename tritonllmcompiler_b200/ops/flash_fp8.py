"""FP8 (e4m3) flash attention forward on B200: the tcgen05 kind::f8f6f4 path.

An extension of the reference's ``flash_attention`` (python/triton_llm/ops/flash_attention.py:
107-133, fp16/bf16 only) to 8-bit inputs with per-tensor scales:
out = softmax(sm_scale * (scale_q q)(scale_k k)^T [top-left causal]) (scale_v v). V is passed
transposed ([B, H, D, Sk], keys contiguous) so that both operands of P V are K-major, the
layout 8-bit UMMA operands take; ``quantize_qkv_e4m3`` produces it. The package root and
``ops`` keep the reference's four exports; import this from here.
"""
from __future__ import annotations

import torch

from tritonllmcompiler_b200 import _lib
from tritonllmcompiler_b200.ops.swiglu_fp8 import quantize_e4m3

E4M3 = torch.float8_e4m3fn


def _strides_ok(t: torch.Tensor) -> bool:
    s = t.stride()
    return s[-1] == 1 and all(x % 16 == 0 for x in s[:-1]) and t.data_ptr() % 16 == 0


def transpose_v_e4m3(v8: torch.Tensor) -> torch.Tensor:
    """[B, H, Sk, D] e4m3 -> V transposed [B, H, D, Sk], stored with its key rows padded to a
    multiple of 16 (the row stride a TMA map needs); the padding is zero and never read."""
    b, h, sk, d = v8.shape
    pad = max(16, (sk + 15) // 16 * 16)
    buf = torch.zeros((b, h, d, pad), dtype=torch.uint8, device=v8.device)
    buf[..., :sk].copy_(v8.view(torch.uint8).transpose(-1, -2))
    return buf.view(E4M3)[..., :sk]


def quantize_qkv_e4m3(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    """Per-tensor e4m3 quantization of [B, H, S, D] q, k, v for ``flash_attention_fp8``.

    Returns (q8, k8, vt8, scale_q, scale_k, scale_v), t ~= t8.float() * scale, with vt8 the
    quantized V transposed ([B, H, D, Sk])."""
    q8, sq = quantize_e4m3(q)
    k8, sk = quantize_e4m3(k)
    v8, sv = quantize_e4m3(v)
    return q8, k8, transpose_v_e4m3(v8), sq, sk, sv


def flash_attention_fp8(q8: torch.Tensor, k8: torch.Tensor, vt8: torch.Tensor, scale_q: float,
                        scale_k: float, scale_v: float, *, causal: bool = False,
                        sm_scale: float | None = None,
                        out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """q8: [B, H, Sq, D], k8: [B, H, Sk, D], vt8: [B, H, D, Sk], all torch.float8_e4m3fn,
    D 64 or 128. Returns a new contiguous [B, H, Sq, D] tensor of out_dtype (fp16 or bf16).
    ``sm_scale`` defaults to D^-0.5, as in ``flash_attention``."""
    assert q8.is_cuda and q8.dim() == 4 and k8.dim() == 4 and vt8.dim() == 4
    assert q8.dtype == E4M3 and k8.dtype == E4M3 and vt8.dtype == E4M3
    b, h, sq, d = q8.shape
    assert d in (64, 128)
    assert k8.shape[:2] == (b, h) and k8.shape[3] == d
    sk = k8.shape[2]
    assert tuple(vt8.shape) == (b, h, d, sk)
    assert out_dtype in _lib.DTYPE_CODES
    assert scale_q > 0 and scale_k > 0 and scale_v > 0
    if sm_scale is None:
        sm_scale = d ** -0.5
    out = torch.empty((b, h, sq, d), device=q8.device, dtype=out_dtype)
    if b == 0 or h == 0 or sq == 0:
        return out
    q8 = q8 if _strides_ok(q8) else q8.contiguous()
    k8 = k8 if _strides_ok(k8) else k8.contiguous()
    if not _strides_ok(vt8):
        vt8 = transpose_v_e4m3(vt8.transpose(-1, -2))
    with _lib.on_device(q8):
        _lib.check(_lib.load().tllm_flash_attn_fp8_fwd(
            q8.data_ptr(), k8.data_ptr(), vt8.data_ptr(), out.data_ptr(), b, h, sq, sk, d,
            _lib.strides(q8), _lib.strides(k8), _lib.strides(vt8), _lib.strides(out),
            float(sm_scale), float(scale_q), float(scale_k), float(scale_v), int(bool(causal)),
            _lib.DTYPE_CODES[out_dtype], _lib.stream_of(q8)))
    return out
