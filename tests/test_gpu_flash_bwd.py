"""FlashAttention backward kernel vs the fp32 oracle (gradients of the reference's forward)."""
import numpy as np
import pytest
import torch

from oracle import flash_bwd_oracle as F
from tritonllmcompiler_b200 import _lib
from tritonllmcompiler_b200.ops.flash_attention import flash_attention
from tritonllmcompiler_b200.ops.flash_backward import (flash_attention_backward, flash_attention_fwd_lse,
                                                       flash_attention_train)

pytestmark = pytest.mark.gpu

# Gradients go through P and dS rounded to the I/O dtype (as the forward's P): tolerance
# per element plus a bound on the relative Frobenius error of each gradient.
TOL = {torch.float16: dict(atol=5e-3, rtol=2e-2, rel=1e-2), torch.bfloat16: dict(atol=3e-2, rtol=5e-2, rel=4e-2)}


def _inputs(seed, b, h, sq, sk, d, dtype):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, h, sq, d, generator=g).to(dtype)
    k = torch.randn(b, h, sk, d, generator=g).to(dtype)
    v = torch.randn(b, h, sk, d, generator=g).to(dtype)
    do = torch.randn(b, h, sq, d, generator=g).to(dtype)
    return q, k, v, do


def _close(got, want, dtype):
    t = TOL[dtype]
    got = got.float().cpu().numpy()
    rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-6)
    assert rel < t["rel"], f"relative error {rel}"
    np.testing.assert_allclose(got, want, atol=t["atol"], rtol=t["rtol"])


@pytest.mark.parametrize("b,h,sq,sk,d,causal,dtype", [
    (1, 2, 256, 256, 128, True, torch.float16),
    (1, 2, 256, 256, 128, False, torch.float16),
    (2, 2, 300, 300, 64, True, torch.float16),
    (1, 1, 128, 384, 128, False, torch.float16),
    (1, 2, 200, 130, 64, True, torch.float16),
    (1, 2, 520, 520, 128, True, torch.bfloat16),
])
def test_backward_matches_oracle(cuda_device, b, h, sq, sk, d, causal, dtype):
    q, k, v, do = _inputs(sq + sk + d, b, h, sq, sk, d, dtype)
    qc, kc, vc, doc = q.cuda(), k.cuda(), v.cuda(), do.cuda()
    o, lse = flash_attention_fwd_lse(qc, kc, vc, causal=causal)
    assert torch.equal(o, flash_attention(qc, kc, vc, causal=causal))
    want_lse = F.forward_lse(q.float().numpy(), k.float().numpy(), causal, d ** -0.5)
    np.testing.assert_allclose(lse.cpu().numpy(), want_lse, atol=2e-3, rtol=1e-4)
    dq, dk, dv = flash_attention_backward(qc, kc, vc, o, lse, doc, causal=causal)
    wq, wk, wv = F.flash_attention_backward(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                            do.float().numpy(), causal=causal,
                                            dtype="bf16" if dtype == torch.bfloat16 else "fp16")
    for got, want in [(dv, wv), (dk, wk), (dq, wq)]:
        _close(got, want, dtype)
    assert _lib.debug_status() == 0


def test_autograd_function(cuda_device):
    q, k, v, do = _inputs(5, 1, 2, 192, 192, 64, torch.float16)
    qc, kc, vc = (t.cuda().requires_grad_() for t in (q, k, v))
    out = flash_attention_train(qc, kc, vc, causal=True)
    out.backward(do.cuda())
    o, lse = flash_attention_fwd_lse(qc.detach(), kc.detach(), vc.detach(), causal=True)
    dq, dk, dv = flash_attention_backward(qc.detach(), kc.detach(), vc.detach(), o, lse, do.cuda(),
                                          causal=True)
    assert torch.equal(qc.grad, dq) and torch.equal(kc.grad, dk) and torch.equal(vc.grad, dv)
