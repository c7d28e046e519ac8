"""Packed variable-length flash attention vs the oracle, and bit-exactly vs the dense kernel
when every sequence has the same length."""
import numpy as np
import pytest
import torch

from oracle import varlen_oracle as V
from tritonllmcompiler_b200 import _lib
from tritonllmcompiler_b200.ops.flash_attention import flash_attention
from tritonllmcompiler_b200.ops.flash_varlen import flash_attention_varlen

pytestmark = pytest.mark.gpu


def _case(seed, lq, lk, h, hkv, d, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    cq = torch.tensor(np.cumsum([0] + lq), dtype=torch.int32)
    ck = torch.tensor(np.cumsum([0] + lk), dtype=torch.int32)
    q = torch.randn(int(cq[-1]), h, d, generator=g).to(dtype)
    k = torch.randn(int(ck[-1]), hkv, d, generator=g).to(dtype)
    v = torch.randn(int(ck[-1]), hkv, d, generator=g).to(dtype)
    return q, k, v, cq, ck


def _check(q, k, v, cq, ck, lq, lk, causal):
    out = flash_attention_varlen(q.cuda(), k.cuda(), v.cuda(), cq.cuda(), ck.cuda(), max(lq),
                                 max(lk), causal=causal)
    ref = V.flash_attention_varlen(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                   cq.numpy(), ck.numpy(), causal=causal,
                                   dtype="bf16" if q.dtype == torch.bfloat16 else "fp16")
    got = out.float().cpu().numpy()
    tol = dict(atol=1e-2, rtol=1e-2) if q.dtype == torch.bfloat16 else dict(atol=1e-3, rtol=1e-2)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    np.testing.assert_allclose(np.nan_to_num(got), np.nan_to_num(ref), **tol)
    assert _lib.debug_status() == 0
    return out


@pytest.mark.parametrize("lq,h,hkv,d,causal,dtype", [
    ([300, 1, 129, 512, 77], 4, 4, 128, True, torch.float16),
    ([300, 1, 129, 512, 77], 4, 4, 128, False, torch.float16),
    ([1000, 256, 33], 8, 2, 128, True, torch.float16),      # GQA
    ([640, 200], 4, 1, 64, True, torch.bfloat16),          # MQA, D 64, bf16
    ([90, 0, 300], 2, 2, 32, True, torch.float16),         # empty sequence, D 32
    ([17, 400], 2, 2, 16, False, torch.float16),           # D 16
])
def test_varlen_matches_oracle(cuda_device, lq, h, hkv, d, causal, dtype):
    q, k, v, cq, ck = _case(sum(lq) + h, lq, lq, h, hkv, d, dtype)
    _check(q, k, v, cq, ck, lq, lq, causal)


def test_varlen_keys_differ_from_queries(cuda_device):
    lq, lk = [100, 300, 5], [260, 130, 0]  # the last sequence has no keys: NaN rows
    q, k, v, cq, ck = _case(7, lq, lk, 4, 2, 128)
    for causal in (False, True):
        _check(q, k, v, cq, ck, lq, lk, causal)


@pytest.mark.parametrize("causal", [False, True])
def test_equal_lengths_are_bit_identical_to_dense(cuda_device, causal):
    B, S, H, D = 3, 700, 8, 128
    q, k, v, cq, ck = _case(11, [S] * B, [S] * B, H, H, D)
    out = flash_attention_varlen(q.cuda(), k.cuda(), v.cuda(), cq.cuda(), ck.cuda(), S, S,
                                 causal=causal)
    dense = lambda t: t.cuda().view(B, S, H, D).permute(0, 2, 1, 3)  # noqa: E731
    ref = flash_attention(dense(q), dense(k), dense(v), causal=causal)
    assert torch.equal(out.view(B, S, H, D).permute(0, 2, 1, 3), ref)


def test_varlen_offsets_past_the_tensor_are_clamped(cuda_device):
    # A cumulative length past the last row is clamped to it, so the last sequence ends at the
    # tensor's end and no store can land outside o.
    q, k, v, cq, ck = _case(13, [64, 64], [64, 64], 2, 2, 64)
    good = flash_attention_varlen(q.cuda(), k.cuda(), v.cuda(), cq.cuda(), ck.cuda(), 64, 64)
    cq_bad = torch.tensor([0, 64, 10_000], dtype=torch.int32)
    ck_bad = torch.tensor([0, 64, 99_999], dtype=torch.int32)
    bad = flash_attention_varlen(q.cuda(), k.cuda(), v.cuda(), cq_bad.cuda(), ck_bad.cuda(), 64, 64)
    assert torch.equal(good, bad)
