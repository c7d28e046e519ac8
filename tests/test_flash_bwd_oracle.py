"""The backward-pass oracle against torch autograd of the reference's forward (CPU, fp32)."""
import numpy as np
import torch

from oracle import flash_bwd_oracle as F
from oracle import ops_oracle as O


def _ref_torch(q, k, v, causal, scale):
    # python/triton_llm/reference/flash_attention.py:12-29 restated in torch, differentiated
    s = (q @ k.transpose(-1, -2)) * scale
    if causal:
        m, n = s.shape[-2:]
        s = s.masked_fill(torch.triu(torch.ones(m, n, dtype=torch.bool), diagonal=1), float("-inf"))
    return torch.softmax(s, dim=-1) @ v


def test_backward_oracle_matches_autograd():
    g = torch.Generator().manual_seed(0)
    for causal, (sq, sk) in [(False, (37, 53)), (True, (40, 40)), (True, (20, 33))]:
        q = torch.randn(2, 3, sq, 16, generator=g, requires_grad=True)
        k = torch.randn(2, 3, sk, 16, generator=g, requires_grad=True)
        v = torch.randn(2, 3, sk, 16, generator=g, requires_grad=True)
        do = torch.randn(2, 3, sq, 16, generator=g)
        _ref_torch(q, k, v, causal, 0.25).backward(do)
        dq, dk, dv = F.flash_attention_backward(q.detach().numpy(), k.detach().numpy(),
                                                v.detach().numpy(), do.numpy(), causal=causal,
                                                sm_scale=0.25, dtype="fp16")
        for got, want in [(dq, q.grad), (dk, k.grad), (dv, v.grad)]:
            np.testing.assert_allclose(got, O.round_to(want.numpy(), "fp16"), atol=2e-3, rtol=1e-2)


def test_lse_oracle_normalises_the_softmax():
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 2, 9, 8)).astype(np.float32)
    k = rng.standard_normal((1, 2, 9, 8)).astype(np.float32)
    lse = F.forward_lse(q, k, causal=True, sm_scale=0.3)
    s = (q @ np.swapaxes(k, -1, -2)) * 0.3 * F.LOG2E
    s = np.where(np.triu(np.ones((9, 9), bool), 1), -np.inf, s)
    np.testing.assert_allclose(np.sum(np.exp2(s - lse[..., None]), axis=-1), 1.0, rtol=1e-5)
