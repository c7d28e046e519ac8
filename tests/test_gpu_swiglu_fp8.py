"""FP8 swiglu kernel vs the swiglu oracle applied to the dequantized e4m3 inputs.

The e4m3 products are exact in fp32, so the kernel differs from the oracle only by the fp32
accumulation order and the final rounding: the fp16 op tolerance applies."""
import numpy as np
import pytest
import torch

from oracle import ops_oracle as O
from tritonllmcompiler_b200 import _lib
from tritonllmcompiler_b200.ops.swiglu_fp8 import quantize_e4m3, swiglu_fp8

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k,out_dtype", [(256, 384, 512, torch.float16), (300, 200, 1040, torch.float16),
                                             (128, 256, 4096, torch.bfloat16), (1, 16, 16, torch.float16)])
def test_fp8_swiglu_matches_oracle(cuda_device, m, n, k, out_dtype):
    g = torch.Generator().manual_seed(m + n + k)
    x = torch.randn(m, k, generator=g)
    w1 = torch.randn(k, n, generator=g) / k ** 0.5
    w3 = torch.randn(k, n, generator=g) / k ** 0.5
    x8, sx = quantize_e4m3(x)
    w18, s1 = quantize_e4m3(w1.t().contiguous())
    w38, s3 = quantize_e4m3(w3.t().contiguous())
    out = swiglu_fp8(x8.cuda(), w18.cuda(), w38.cuda(), sx, s1, s3, out_dtype)
    xd = x8.float().numpy() * np.float32(sx)
    w1d = (w18.float().numpy() * np.float32(s1)).T
    w3d = (w38.float().numpy() * np.float32(s3)).T
    # the kernel scales the accumulators: silu(sx*s1 * sum(x8*w8)) * (sx*s3 * sum(x8*w8))
    ref = O.swiglu(xd, w1d, w3d, dtype="bf16" if out_dtype == torch.bfloat16 else "fp16")
    tol = dict(atol=1e-2, rtol=1e-2) if out_dtype == torch.bfloat16 else dict(atol=2e-3, rtol=1e-2)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, **tol)
    assert _lib.debug_status() == 0


def test_fp8_swiglu_strided_output_rows(cuda_device):
    g = torch.Generator().manual_seed(3)
    x8, sx = quantize_e4m3(torch.randn(130, 256, generator=g))
    w18, s1 = quantize_e4m3(torch.randn(144, 256, generator=g) / 16)
    w38, s3 = quantize_e4m3(torch.randn(144, 256, generator=g) / 16)
    a = swiglu_fp8(x8.cuda(), w18.cuda(), w38.cuda(), sx, s1, s3)
    big = torch.zeros(130, 512, dtype=torch.uint8).to(torch.float8_e4m3fn)
    big[:, :256] = x8
    b = swiglu_fp8(big.cuda()[:, :256], w18.cuda(), w38.cuda(), sx, s1, s3)
    assert torch.equal(a, b)


@pytest.mark.parametrize("m,n,k,out_dtype,variants", [
    (256, 128, 128, torch.float16, (1, 2)),
    (300, 200, 1040, torch.float16, (1, 2)),     # ragged M, N and K: zero-filled edge tiles
    (128, 384, 512, torch.bfloat16, (1, 2)),     # forced pair with the second CTA's rows past M
    (1000, 640, 528, torch.bfloat16, (1, 2, 0)),
    (260, 100, 256, torch.float16, (1, 2, 0)),    # ldo = 100: the scalar-store epilogue
    (256, 48, 16, torch.bfloat16, (1, 2)),        # K = 16: one k block, mostly zero-filled
    (4096, 1024, 4096, torch.float16, (1, 2, 0)),
])
def test_fp8_swiglu_kernel_variants_agree(cuda_device, m, n, k, out_dtype, variants):
    """The CTA-pair kernel (tcgen05.mma.cta_group::2, two SMs per 256 x 128 tile) and the
    one-CTA kernel accumulate every output element in the same K order: bit-identical; the
    automatic choice (0) takes the pair kernel from M >= 256."""
    g = torch.Generator().manual_seed(m * 7 + n + k)
    x8, sx = quantize_e4m3(torch.randn(m, k, generator=g))
    w18, s1 = quantize_e4m3(torch.randn(n, k, generator=g) / k ** 0.5)
    w38, s3 = quantize_e4m3(torch.randn(n, k, generator=g) / k ** 0.5)
    x8, w18, w38 = x8.cuda(), w18.cuda(), w38.cuda()
    outs = []
    for variant in variants:
        o = torch.full((m, n), float("nan"), dtype=out_dtype, device="cuda")
        _lib.check(_lib.load().tllm_swiglu_fp8_variant(
            x8.data_ptr(), w18.data_ptr(), w38.data_ptr(), o.data_ptr(), m, n, k, k, k, k, n,
            sx, s1, s3, _lib.DTYPE_CODES[out_dtype], variant,
            torch.cuda.current_stream().cuda_stream))
        outs.append(o)
    for o in outs[1:]:
        assert torch.equal(outs[0], o)
    assert not torch.isnan(outs[0]).any()
    assert torch.equal(outs[0], swiglu_fp8(x8, w18, w38, sx, s1, s3, out_dtype))
    assert _lib.debug_status() == 0
