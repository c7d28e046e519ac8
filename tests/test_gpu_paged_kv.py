"""Paged-KV append kernels vs the oracle (bit-exact: they only move and round bytes) and vs
the library's own rmsnorm_rope (bit-exact: same row arithmetic)."""
import numpy as np
import pytest
import torch

import tritonllmcompiler_b200 as T
from oracle import ops_oracle as O
from oracle import paged_kv_oracle as P
from tritonllmcompiler_b200 import _lib
from tritonllmcompiler_b200.ops import paged_kv as K

pytestmark = pytest.mark.gpu


def _case(seed, B, Tn, H, D, bs, start, dtype=torch.float16, extra_blocks=2):
    g = torch.Generator().manual_seed(seed)
    start = torch.tensor(start, dtype=torch.int32)
    ends = start + Tn
    nb = [(int(e) + bs - 1) // bs for e in ends]
    pool = sum(nb) + extra_blocks
    perm = torch.randperm(pool, generator=g)
    bt = torch.zeros(B, max(nb), dtype=torch.int32)
    i = 0
    for b, n in enumerate(nb):
        bt[b, :n] = perm[i:i + n]
        i += n
    kc = torch.randn(pool, bs, H, D, generator=g).to(dtype)
    vc = torch.randn(pool, bs, H, D, generator=g).to(dtype)
    kn = torch.randn(B, Tn, H, D, generator=g).to(dtype)
    vn = torch.randn(B, Tn, H, D, generator=g).to(dtype)
    return kn, vn, kc, vc, bt, start


@pytest.mark.parametrize("B,Tn,H,D,bs,dtype", [(3, 5, 8, 128, 16, torch.float16),
                                                (2, 33, 3, 64, 32, torch.bfloat16),
                                                (4, 1, 6, 32, 16, torch.float16),
                                                (1, 70, 2, 16, 64, torch.float16)])
def test_append_matches_oracle_exactly(cuda_device, B, Tn, H, D, bs, dtype):
    start = [(7 * b + 3) % 50 for b in range(B)]
    kn, vn, kc, vc, bt, sp = _case(B * 100 + Tn, B, Tn, H, D, bs, start, dtype)
    n_new = torch.tensor([max(0, Tn - b) for b in range(B)], dtype=torch.int32)
    kcg, vcg = kc.cuda(), vc.cuda()
    K.paged_kv_append(kn.cuda(), vn.cuda(), kcg, vcg, bt.cuda(), sp.cuda(), n_new.cuda(), block_size=bs)
    wk, wv = P.paged_kv_append(kn.float().numpy(), vn.float().numpy(), kc.float().numpy(),
                               vc.float().numpy(), bt.numpy(), sp.numpy(), n_new.numpy(), block_size=bs)
    np.testing.assert_array_equal(kcg.float().cpu().numpy(), wk)
    np.testing.assert_array_equal(vcg.float().cpu().numpy(), wv)
    assert _lib.debug_status() == 0


def test_append_strided_new_tokens(cuda_device):
    kn, vn, kc, vc, bt, sp = _case(5, 2, 9, 4, 64, 16, [0, 12])
    big = torch.randn(2, 9, 8, 64).half()
    big[:, :, ::2] = kn  # k_new as a strided view (every other head)
    kcg, vcg = kc.cuda(), vc.cuda()
    K.paged_kv_append(big.cuda()[:, :, ::2], vn.cuda(), kcg, vcg, bt.cuda(), sp.cuda(), block_size=16)
    wk, _ = P.paged_kv_append(kn.float().numpy(), vn.float().numpy(), kc.float().numpy(),
                              vc.float().numpy(), bt.numpy(), sp.numpy(), None, block_size=16)
    np.testing.assert_array_equal(kcg.float().cpu().numpy(), wk)


@pytest.mark.parametrize("D,dtype", [(128, torch.float16), (64, torch.bfloat16), (32, torch.float16)])
def test_append_rope_equals_rmsnorm_rope_then_append(cuda_device, D, dtype):
    B, Tn, H, bs = 3, 11, 8, 16
    start = [0, 9, 30]
    kn, vn, kc, vc, bt, sp = _case(D, B, Tn, H, D, bs, start, dtype)
    g = torch.Generator().manual_seed(D + 1)
    P_rows = 64
    w = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    pos = torch.arange(P_rows, dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2).float() / D))
    emb = torch.cat([torch.outer(pos, inv)] * 2, dim=-1)
    cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
    kcg, vcg = kc.cuda(), vc.cuda()
    K.paged_kv_append_rope(kn.cuda(), vn.cuda(), w.cuda(), cos.cuda(), sin.cuda(), kcg, vcg,
                           bt.cuda(), sp.cuda(), block_size=bs)
    # The library's own rmsnorm_rope on each sequence's rows (cos/sin at absolute positions),
    # then a plain append: bit-identical.
    kc2, vc2 = kc.cuda(), vc.cuda()
    rot = torch.empty_like(kn).cuda()
    for b in range(B):
        p = sp[b].item() + torch.arange(Tn)
        rot[b:b + 1] = T.rmsnorm_rope(kn[b:b + 1].cuda(), w.cuda(), cos[p].cuda(), sin[p].cuda())
    K.paged_kv_append(rot, vn.cuda(), kc2, vc2, bt.cuda(), sp.cuda(), block_size=bs)
    assert torch.equal(kcg, kc2) and torch.equal(vcg, vc2)
    # and against the oracle within the op tolerance
    wk, wv = P.paged_kv_append_rope(kn.float().numpy(), vn.float().numpy(), w.float().numpy(),
                                    cos.float().numpy(), sin.float().numpy(), kc.float().numpy(),
                                    vc.float().numpy(), bt.numpy(), sp.numpy(), block_size=bs,
                                    dtype="bf16" if dtype == torch.bfloat16 else "fp16")
    tol = dict(atol=1e-2, rtol=1e-2) if dtype == torch.bfloat16 else dict(atol=1e-3, rtol=1e-2)
    np.testing.assert_allclose(kcg.float().cpu().numpy(), wk, **tol)
    np.testing.assert_array_equal(vcg.float().cpu().numpy(), wv)
    assert _lib.debug_status() == 0


def test_append_bad_positions_are_skipped_and_flagged(cuda_device):
    kn, vn, kc, vc, bt, sp = _case(9, 2, 4, 2, 64, 16, [0, 0])
    bt[1, 0] = 10_000  # outside the pool
    sp_bad = torch.tensor([0, 0], dtype=torch.int32)
    kcg, vcg = kc.cuda(), vc.cuda()
    K.paged_kv_append(kn.cuda(), vn.cuda(), kcg, vcg, bt.cuda(), sp_bad.cuda(), block_size=16)
    torch.cuda.synchronize()
    assert _lib.debug_status() == 0x200
    # sequence 0 was written, sequence 1 touched nothing
    got = kcg.cpu()
    assert torch.equal(got[bt[0, 0], :4], kn[0])
    mask = torch.ones(kc.shape[0], dtype=torch.bool)
    mask[bt[0, 0]] = False
    assert torch.equal(got[mask], kc[mask])
    # a start position past the table is skipped too
    kcg2 = kc.cuda()
    K.paged_kv_append(kn.cuda(), vn.cuda(), kcg2, vc.cuda(), bt.cuda(),
                      torch.tensor([1000, 0], dtype=torch.int32).cuda(), block_size=16)
    torch.cuda.synchronize()
    assert _lib.debug_status() == 0x200
    assert _lib.debug_status() == 0


# ------------------------------------------------------------ multi-token GQA paged attention
def _prefill_case(seed, lens, hkv, g, sq, d, bs, dtype=torch.float16, extra=3):
    gen = torch.Generator().manual_seed(seed)
    lens = torch.tensor(lens, dtype=torch.int32)
    nb = [max(1, (int(n) + bs - 1) // bs) for n in lens]
    pool = sum(nb) + extra
    perm = torch.randperm(pool, generator=gen)
    bt = torch.zeros(len(lens), max(nb), dtype=torch.int32)
    i = 0
    for b, n in enumerate(nb):
        bt[b, :n] = perm[i:i + n]
        i += n
    kc = torch.randn(pool, bs, hkv, d, generator=gen).to(dtype)
    vc = torch.randn(pool, bs, hkv, d, generator=gen).to(dtype)
    q = torch.randn(len(lens), hkv * g, sq, d, generator=gen).to(dtype)
    return q, kc, vc, bt, lens


def _prefill_check(q, kc, vc, bt, lens, bs, causal=True):
    out = K.paged_attention_prefill(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), lens.cuda(),
                                    block_size=bs, causal=causal)
    ref = P.paged_attention_prefill(q.float().numpy(), kc.float().numpy(), vc.float().numpy(),
                                    bt.numpy(), lens.numpy(), block_size=bs, causal=causal,
                                    dtype="bf16" if q.dtype == torch.bfloat16 else "fp16")
    got = out.float().cpu().numpy()
    tol = dict(atol=1e-2, rtol=1e-2) if q.dtype == torch.bfloat16 else dict(atol=1e-3, rtol=1e-2)
    assert got.shape == ref.shape
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    np.testing.assert_allclose(np.nan_to_num(got), np.nan_to_num(ref), **tol)
    assert _lib.debug_status() == 0
    return out


@pytest.mark.parametrize("lens,hkv,g,sq,d,bs", [
    ([37, 300, 1, 128], 4, 1, 1, 128, 16),      # reference decode shape
    ([500, 129, 64], 2, 4, 1, 128, 16),         # GQA decode
    ([260, 40, 999], 2, 4, 4, 128, 32),         # multi-token GQA (16 rows per tile)
    ([77, 513], 1, 8, 7, 64, 16),               # 56 rows per tile
    ([1000, 333], 2, 4, 32, 128, 64),           # 128 rows per tile
    ([700, 300], 1, 2, 200, 128, 16),           # prefill: two token tiles per head
    ([5, 130, 17], 3, 2, 5, 32, 16),            # short contexts, D 32
    ([64, 1, 3], 2, 1, 3, 16, 16),              # D 16, contexts shorter than the new tokens
    # at most 16 query rows per KV head (D 64/128): the grouped-query split kernel
    ([2, 1, 300, 4], 2, 2, 4, 128, 16),         # contexts shorter than the new tokens
    ([37, 500], 4, 1, 6, 64, 16),               # one head per KV head, 6 new tokens
    ([100, 2000], 1, 8, 2, 64, 32),             # 16 rows at D 64
    ([3000, 7000, 20], 2, 16, 1, 128, 16),      # 16 query heads per KV head, one token
    ([5000, 129], 1, 5, 3, 128, 64),            # 15 rows, split keys
])
def test_prefill_matches_oracle(cuda_device, lens, hkv, g, sq, d, bs):
    q, kc, vc, bt, cl = _prefill_case(sum(lens) + sq, lens, hkv, g, sq, d, bs)
    _prefill_check(q, kc, vc, bt, cl, bs)


def test_prefill_non_causal_and_bf16(cuda_device):
    q, kc, vc, bt, cl = _prefill_case(3, [150, 900], 2, 3, 6, 128, 16, dtype=torch.bfloat16)
    _prefill_check(q, kc, vc, bt, cl, 16, causal=False)
    # 15 and 4 query rows per KV head: the grouped-query split kernel
    q, kc, vc, bt, cl = _prefill_case(4, [150, 4900, 3], 2, 3, 5, 128, 16, dtype=torch.bfloat16)
    _prefill_check(q, kc, vc, bt, cl, 16, causal=False)
    q, kc, vc, bt, cl = _prefill_case(5, [2, 77], 1, 2, 2, 64, 16, dtype=torch.bfloat16)
    _prefill_check(q, kc, vc, bt, cl, 16, causal=False)


def test_prefill_split_kv_long_context(cuda_device):
    # Few items and long contexts: the keys are split over several CTAs and merged.
    q, kc, vc, bt, cl = _prefill_case(11, [8000, 2500], 1, 4, 2, 128, 16)
    assert _lib.load().tllm_paged_prefill_workspace_size(2, 4, 1, 2, 128, 16, bt.shape[1]) > 0
    _prefill_check(q, kc, vc, bt, cl, 16)


@pytest.mark.parametrize("lens,hkv,g,d,dtype", [([8000, 2500], 1, 4, 128, torch.float16),   # splits
                                                ([300, 1, 77, 4096], 2, 8, 64, torch.float16),
                                                ([513, 900], 4, 2, 128, torch.bfloat16),
                                                ([0, 40, 7000], 2, 4, 128, torch.float16),
                                                ([1, 2, 3000], 8, 4, 64, torch.bfloat16),
                                                ([5000, 33, 0], 3, 5, 128, torch.float16)])
def test_gqa_single_token_decode(cuda_device, lens, hkv, g, d, dtype):
    # One new token per sequence and several query heads per KV head (the grouped-query split
    # kernel at D 64 and 128, with 2 to 8 query rows); an empty context gives NaN as in the
    # reference.
    q, kc, vc, bt, cl = _prefill_case(sum(lens) + g, lens, hkv, g, 1, d, 16, dtype)
    _prefill_check(q, kc, vc, bt, cl, 16)


def test_prefill_empty_context_is_nan(cuda_device):
    q, kc, vc, bt, cl = _prefill_case(12, [0, 40], 2, 2, 3, 64, 16)
    out = _prefill_check(q, kc, vc, bt, cl, 16)
    assert torch.isnan(out[0]).all()


def test_prefill_unwritten_cache_tail_never_reaches_the_output(cuda_device):
    # Cache slots past each context hold NaN (unwritten memory); the kernel must not read
    # them into the accumulator.
    q, kc, vc, bt, cl = _prefill_case(13, [20, 150], 2, 2, 2, 128, 16)
    for b, n in enumerate(cl.tolist()):
        nb = (n + 15) // 16
        last = bt[b, nb - 1]
        kc[last, n % 16 or 16:] = float("nan")
        vc[last, n % 16 or 16:] = float("nan")
    out = _prefill_check(q, kc, vc, bt, cl, 16)
    assert torch.isfinite(out).all()


def test_prefill_one_token_equals_decode_kernel(cuda_device):
    q, kc, vc, bt, cl = _prefill_case(14, [1000, 37, 4096, 513], 8, 1, 1, 128, 16)
    a = K.paged_attention_prefill(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), cl.cuda(), block_size=16)
    b = T.paged_attention(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), cl.cuda(), block_size=16)
    assert torch.equal(a, b)  # the same decode kernel


def test_prefill_bad_block_entry_is_flagged(cuda_device):
    q, kc, vc, bt, cl = _prefill_case(15, [40, 40], 1, 2, 1, 64, 16)
    bt[1, 1] = -5
    K.paged_attention_prefill(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), cl.cuda(), block_size=16)
    torch.cuda.synchronize()
    assert _lib.debug_status() == 0x200


def test_decode_step_composes(cuda_device):
    """One decode step of a GQA layer: RoPE'd K and V appended to the cache, then attention of
    the new tokens (q through rmsnorm_rope) over the whole context."""
    B, hkv, g, sq, d, bs = 2, 2, 4, 3, 128, 16
    old = torch.tensor([45, 100], dtype=torch.int32)
    q, kc, vc, bt, _ = _prefill_case(16, (old + sq).tolist(), hkv, g, sq, d, bs)
    gen = torch.Generator().manual_seed(17)
    kn = torch.randn(B, sq, hkv, d, generator=gen).half()
    vn = torch.randn(B, sq, hkv, d, generator=gen).half()
    w = (1 + 0.1 * torch.randn(d, generator=gen)).half()
    pos = torch.arange(256, dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, d, 2).float() / d))
    emb = torch.cat([torch.outer(pos, inv)] * 2, dim=-1)
    cos, sin = emb.cos().half(), emb.sin().half()
    kcg, vcg = kc.cuda(), vc.cuda()
    K.paged_kv_append_rope(kn.cuda(), vn.cuda(), w.cuda(), cos.cuda(), sin.cuda(), kcg, vcg,
                           bt.cuda(), old.cuda(), block_size=bs)
    cl = old + sq
    out = K.paged_attention_prefill(q.cuda(), kcg, vcg, bt.cuda(), cl.cuda(), block_size=bs)
    k2, v2 = P.paged_kv_append_rope(kn.float().numpy(), vn.float().numpy(), w.float().numpy(),
                                    cos.float().numpy(), sin.float().numpy(), kc.float().numpy(),
                                    vc.float().numpy(), bt.numpy(), old.numpy(), block_size=bs)
    ref = P.paged_attention_prefill(q.float().numpy(), k2, v2, bt.numpy(), cl.numpy(), block_size=bs)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-3, rtol=1e-2)
