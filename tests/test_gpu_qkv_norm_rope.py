"""Fused QKV projection + RMSNorm + RoPE vs the oracle (projection, rounding, rmsnorm_rope)."""
import numpy as np
import pytest
import torch

from oracle import qkv_oracle as Q
from tritonllmcompiler_b200 import _lib
from tritonllmcompiler_b200.ops.qkv_norm_rope import qkv_norm_rope

pytestmark = pytest.mark.gpu


def _tables(p, d, dtype):
    pos = torch.arange(p, dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, d, 2).float() / d))
    emb = torch.cat([torch.outer(pos, inv)] * 2, dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


@pytest.mark.parametrize("m,k,hq,hkv,dtype", [(256, 512, 4, 2, torch.float16), (300, 1024, 8, 1, torch.float16),
                                              (64, 256, 3, 1, torch.bfloat16), (130, 4096, 2, 2, torch.float16),
                                              # more tiles than SMs: the partial last wave runs as
                                              # one-head tiles (11 heads: one of them is past the end)
                                              (2048, 512, 16, 4, torch.float16),
                                              (4096, 256, 7, 2, torch.bfloat16)])
def test_qkv_norm_rope_matches_oracle(cuda_device, m, k, hq, hkv, dtype):
    g = torch.Generator().manual_seed(m + k)
    n = (hq + 2 * hkv) * 128
    x = torch.randn(m, k, generator=g).to(dtype)
    w = (torch.randn(k, n, generator=g) / k ** 0.5).to(dtype)
    wq = (1 + 0.1 * torch.randn(128, generator=g)).to(dtype)
    wk = (1 + 0.1 * torch.randn(128, generator=g)).to(dtype)
    cos, sin = _tables(1024, 128, dtype)
    positions = torch.randint(0, 1024, (m,), generator=g, dtype=torch.int32)
    out = qkv_norm_rope(x.cuda(), w.cuda(), wq.cuda(), wk.cuda(), cos.cuda(), sin.cuda(), positions.cuda(),
                        num_q_heads=hq, num_kv_heads=hkv)
    ref = Q.qkv_norm_rope(x.float().numpy(), w.float().numpy(), wq.float().numpy(), wk.float().numpy(),
                          cos.float().numpy(), sin.float().numpy(), positions.numpy(), num_q_heads=hq,
                          num_kv_heads=hkv, dtype="bf16" if dtype == torch.bfloat16 else "fp16")
    got = out.float().cpu().numpy()
    # The projection's fp32 accumulation order may flip a rounding of the stored projection
    # by one ulp, which the norm carries forward: op tolerance.
    tol = dict(atol=2e-2, rtol=2e-2) if dtype == torch.bfloat16 else dict(atol=3e-3, rtol=1e-2)
    np.testing.assert_allclose(got, ref, **tol)
    assert _lib.debug_status() == 0
