"""FP8 (e4m3) flash attention vs the oracle on the dequantized inputs.

The kernel rounds P to e4m3 before P V (a relative error of at most 2^-4 per probability),
so each output element is checked against the oracle's own bound for that rounding,
2^-4 * (softmax @ |v|), plus 2^-9 * max|v| for probabilities in e4m3's subnormal range and
the output rounding (2^-10 relative for fp16, 2^-7 for bf16)."""
import numpy as np
import pytest
import torch

from oracle import fp8_attn_oracle as F
from tests import _golden as G
from tritonllmcompiler_b200 import _lib
from tritonllmcompiler_b200.ops.flash_fp8 import (flash_attention_fp8, quantize_qkv_e4m3,
                                                  transpose_v_e4m3)

pytestmark = pytest.mark.gpu


def _inputs(seed, b, h, sq, sk, d):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, h, sq, d, generator=g)
    k = torch.randn(b, h, sk, d, generator=g)
    v = torch.randn(b, h, sk, d, generator=g)
    return q, k, v


def _check(got, q8, k8, v8, scales, causal, out_dtype, heads=None):
    """got: kernel output [B, H, Sq, D] (cpu float32); heads: (b, h) pairs to compare (all if
    None)."""
    sq_, sk_, sv_ = scales
    pairs = heads or [(b, h) for b in range(q8.shape[0]) for h in range(q8.shape[1])]
    rel_out = 2.0 ** -10 if out_dtype == torch.float16 else 2.0 ** -7
    for b, h in pairs:
        qq, kk, vv = (t[b:b + 1, h:h + 1].float().numpy() for t in (q8, k8, v8))
        ref = F.flash_attention_fp8(qq, kk, vv, sq_, sk_, sv_, causal=causal)
        bound = F.error_bound(qq, kk, vv, sq_, sk_, sv_, causal=causal)
        g = got[b:b + 1, h:h + 1]
        assert np.array_equal(np.isnan(g), np.isnan(ref))
        ok = ~np.isnan(ref)
        vmax = float(np.abs(vv).max()) * sv_ if vv.size else 0.0
        tol = bound + 2.0 ** -9 * vmax + rel_out * np.abs(ref) + 1e-6
        err = np.abs(g - ref)
        assert np.all(err[ok] <= tol[ok]), f"head ({b},{h}): max excess {(err - tol)[ok].max()}"


@pytest.mark.parametrize("b,h,sq,sk,d,causal,out_dtype", [
    (1, 2, 256, 256, 128, True, torch.float16),
    (2, 3, 300, 300, 128, False, torch.float16),
    (1, 2, 129, 700, 128, True, torch.float16),   # Sq != Sk, ragged tiles
    (1, 1, 640, 77, 128, False, torch.bfloat16),  # Sk below one tile, not a multiple of 16
    (2, 2, 384, 384, 64, True, torch.float16),
    (1, 2, 1, 1000, 64, False, torch.bfloat16),
])
def test_fp8_flash_matches_oracle(cuda_device, b, h, sq, sk, d, causal, out_dtype):
    q, k, v = _inputs(b * 1000 + sq + sk + d, b, h, sq, sk, d)
    q8, k8, vt8, s1, s2, s3 = quantize_qkv_e4m3(q, k, v)
    out = flash_attention_fp8(q8.cuda(), k8.cuda(), vt8.cuda(), s1, s2, s3, causal=causal,
                              out_dtype=out_dtype)
    assert out.dtype == out_dtype and out.shape == (b, h, sq, d)
    v8 = vt8.transpose(-1, -2)
    _check(out.float().cpu().numpy(), q8, k8, v8, (s1, s2, s3), causal, out_dtype)
    assert _lib.debug_status() == 0


def test_fp8_flash_strided_inputs(cuda_device):
    # q and k as views into wider buffers (strides multiples of 16), V transposed given as a
    # view whose key stride is not a multiple of 16 (the wrapper repacks it).
    q, k, v = _inputs(7, 1, 4, 200, 260, 128)
    q8, k8, vt8, s1, s2, s3 = quantize_qkv_e4m3(q, k, v)
    qw = torch.zeros(1, 4, 200, 256, dtype=torch.uint8).view(q8.dtype)
    qw.view(torch.uint8)[..., :128].copy_(q8.view(torch.uint8))
    kw = torch.zeros(1, 4, 260, 144, dtype=torch.uint8).view(k8.dtype)
    kw.view(torch.uint8)[..., 16:].copy_(k8.view(torch.uint8))
    v8 = vt8.transpose(-1, -2)
    vt_odd = torch.zeros(1, 4, 128, 261, dtype=torch.uint8)
    vt_odd[..., :260].copy_(v8.view(torch.uint8).transpose(-1, -2))
    out = flash_attention_fp8(qw.cuda()[..., :128], kw.cuda()[..., 16:],
                              vt_odd.cuda().view(q8.dtype)[..., :260], s1, s2, s3, causal=True)
    _check(out.float().cpu().numpy(), q8, k8, v8, (s1, s2, s3), True, torch.float16)


def test_fp8_flash_scale_v_is_exact(cuda_device):
    # The output is (P V) / l times scale_v: doubling scale_v doubles it bit for bit (outside
    # fp16's subnormal range, where the output rounding grid does not scale).
    q, k, v = _inputs(11, 1, 4, 512, 512, 128)
    q8, k8, vt8, s1, s2, s3 = quantize_qkv_e4m3(q, k, v)
    q8, k8, vt8 = q8.cuda(), k8.cuda(), vt8.cuda()
    a = flash_attention_fp8(q8, k8, vt8, s1, s2, s3, causal=True)
    b2 = flash_attention_fp8(q8, k8, vt8, s1, s2, 2 * s3, causal=True)
    G.assert_doubled_exactly(a, b2)


def test_fp8_flash_empty_keys_is_nan(cuda_device):
    # No keys: 0/0, as flash_attention (k is an empty view of a real buffer).
    q, k, v = _inputs(3, 1, 1, 64, 16, 128)
    q8, k8, vt8, s1, s2, s3 = quantize_qkv_e4m3(q, k, v)
    k8 = k8.cuda()[:, :, :0]
    out = flash_attention_fp8(q8.cuda(), k8, transpose_v_e4m3(k8), s1, s2, s3)
    assert torch.isnan(out).all()


def test_fp8_flash_full_size_sampled_heads(cuda_device):
    # The bench shape [4, 32, 4096, 128] causal; eight (b, h) heads compared with the oracle.
    torch.manual_seed(0)
    q, k, v = (torch.randn(4, 32, 4096, 128, device="cuda") for _ in range(3))
    q8, k8, vt8, s1, s2, s3 = quantize_qkv_e4m3(q, k, v)
    out = flash_attention_fp8(q8, k8, vt8, s1, s2, s3, causal=True)
    got = out.float().cpu().numpy()
    v8 = vt8.transpose(-1, -2).cpu()
    _check(got, q8.cpu(), k8.cpu(), v8, (s1, s2, s3), True, torch.float16,
           heads=[(0, 0), (0, 31), (1, 7), (2, 16), (3, 5), (3, 31), (1, 20), (2, 2)])


def test_fp8_flash_rejects_bad_head_dim(cuda_device):
    q8 = torch.zeros(1, 1, 16, 96, dtype=torch.uint8, device="cuda").view(torch.float8_e4m3fn)
    with pytest.raises(AssertionError):
        flash_attention_fp8(q8, q8, q8.transpose(-1, -2), 1.0, 1.0, 1.0)
